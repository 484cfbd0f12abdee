// Backward of the stateful fused GDN-2 scan: dbl_gdn_training_scan_backward.
//
// Replaces delta_kernels' gdn_training_backward (crates/kernels/src/gdn_training_ops.rs:95-127,
// kernel gdn_training.rs:117-284): the vector-Jacobian product of gdn_training_scan for the loss
//     L = sum g_out . out + sum g_fin . final_state + sum g_score . scores.
// The reference backward reads the checkpoints and per-token edits its forward saved; this entry
// point recomputes them into the caller's workspace, so it needs only the forward's inputs.
//
// One CTA per (b, h); thread j owns value column j, as in the forward.
//   pass 1  forward over all tokens, storing the state at every chunk start (checkpoints);
//   pass 2  for each chunk from the last: replay it from its checkpoint, storing each token's
//           previous state (workspace) and edit and |edit| (shared memory), then walk it in
//           reverse with the adjoint column A[., j] in registers:
//             dd_j = g_score |k| edit_j / |edit| + sum_i k_i A_ij     (after A += q dy^T)
//             dq_i = sum_j (bar_ij + k_i edit_j) dy_j,   bar = reset ? 0 : alpha (.) S_prev
//             dk_i = sum_j (A_ij edit_j - erase_i bar_ij dd_j) + g_score |edit| k_i / |k|
//             de_i = -sum_j k_i bar_ij dd_j,   dv_j = dd_j write_j,   dw_j = dd_j v_j
//             dbar = A - erase (.) k dd^T;  reset: A = 0;  else d alpha_i = sum_j dbar_ij S_prev_ij,
//             A = alpha (.) dbar.
// The sums over j use a warp butterfly reduce-scatter (lane L ends with the sum for index L of a
// block of 32) and one shared-memory pass across warps.  f32 throughout, as the reference.
#include <cuda_bf16.h>

#include <algorithm>

#include "common.cuh"

namespace dbl {
namespace {

constexpr unsigned FULL = 0xffffffffu;
constexpr int MAXC = 16;  // largest checkpoint chunk (the reference's 1..=16)

struct BwdParams {
    int B, T, H, K, V, C, nch;
    const float *q, *k, *v, *alpha, *erase, *write, *valid, *reset, *initial;
    const float *g_out, *g_fin, *g_score;
    float *dq, *dk, *dv, *dalpha, *derase, *dwrite, *dinitial;
    float *ck;  // [B*H][nch][K][V] chunk-start states
    float *rp;  // [B*H][C][K][V]   previous state of each token of the chunk being reversed
};

// Sum over the 32 lanes of vals[0..32): afterwards lane L's vals[0] holds the sum for index L.
__device__ __forceinline__ void reduce_scatter32(float (&vals)[32], int lane) {
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
        const bool upper = (lane & o) != 0;
#pragma unroll
        for (int x = 0; x < o; ++x) {
            const float send = upper ? vals[x] : vals[x + o];
            const float keep = upper ? vals[x + o] : vals[x];
            vals[x] = keep + __shfl_xor_sync(FULL, send, o);
        }
    }
}

template <int KMAX>
__global__ void __launch_bounds__(256) training_backward_kernel(const BwdParams p) {
    constexpr int NKB = KMAX / 32;  // 32-wide blocks of key channels
    // the staged chunk: k, alpha, erase, q of its tokens and their masks; per-warp partials
    __shared__ float sk[MAXC][KMAX], sa[MAXC][KMAX], se[MAXC][KMAX], sq[MAXC][KMAX];
    __shared__ float sen[MAXC][8];        // per-warp partial |edit|^2
    __shared__ float red[2][8][4][KMAX];  // per-warp sums dq, dk, dalpha, derase (double-buffered)
    __shared__ int sact[MAXC], srst[MAXC];
    // per column: write * v and the edit of each token of the chunk, [MAXC][blockDim] (dynamic);
    // thread j reads and writes only column j
    extern __shared__ float dyn[];
    float* swv = dyn;
    float* sxe = dyn + MAXC * blockDim.x;

    const int bh = blockIdx.x;
    const int b = bh / p.H, h = bh - b * p.H;
    const int j = threadIdx.x, nthr = blockDim.x;
    const int warp = j >> 5, lane = j & 31, nwarps = nthr >> 5;
    const bool col = j < p.V;
    const int K = p.K, V = p.V, T = p.T, H = p.H;
    const size_t sbase = ((size_t)b * H + h) * K * V;
    auto tok = [&](int t) { return ((size_t)b * T + t) * H + h; };  // token row index

    // stages the n tokens from t0 (k, alpha, erase and, for the reverse, q) with one pair of
    // barriers: every load of the chunk is in flight at once
    auto stage = [&](int t0, int n, bool with_q) {
        __syncthreads();
        for (int x = j; x < n * KMAX; x += nthr) {
            const int r = x / KMAX, i = x - r * KMAX;
            const bool in = i < K;
            const size_t g = tok(t0 + r) * K + i;
            sk[r][i] = in ? p.k[g] : 0.f;
            sa[r][i] = in ? p.alpha[g] : 0.f;
            se[r][i] = in ? p.erase[g] : 0.f;
            if (with_q) sq[r][i] = in ? p.q[g] : 0.f;
        }
        if (j < n) {
            sact[j] = p.valid[(size_t)b * T + t0 + j] != 0.f;
            srst[j] = p.reset[(size_t)b * T + t0 + j] != 0.f;
        }
        __syncthreads();
    };
    // write * v of this column for the chunk's tokens into swv: all loads issued, then stored
    auto load_wv = [&](int t0, int n) {
        float w[MAXC], x[MAXC];
#pragma unroll
        for (int r = 0; r < MAXC; ++r) {
            w[r] = (col && r < n) ? p.write[tok(t0 + r) * V + j] : 0.f;
            x[r] = (col && r < n) ? p.v[tok(t0 + r) * V + j] : 0.f;
        }
#pragma unroll
        for (int r = 0; r < MAXC; ++r) swv[r * nthr + j] = w[r] * x[r];
    };
    // one forward step of this column; returns the edit x
    auto step = [&](float (&S)[KMAX], int r, float wv) {
        if (!sact[r]) return 0.f;
        const bool rst = srst[r];
        float x = wv;
#pragma unroll
        for (int i = 0; i < KMAX; ++i) {
            const float bar = rst ? 0.f : sa[r][i] * S[i];
            x -= se[r][i] * sk[r][i] * bar;
            S[i] = bar;
        }
#pragma unroll
        for (int i = 0; i < KMAX; ++i) S[i] = fmaf(sk[r][i], x, S[i]);
        return x;
    };

    // ---------------------------------------------------------------- pass 1: checkpoints
    float S[KMAX];
#pragma unroll
    for (int i = 0; i < KMAX; ++i) S[i] = (col && i < K && p.initial) ? p.initial[sbase + (size_t)i * V + j] : 0.f;
    for (int c = 0; c < p.nch; ++c) {
        const int t0 = c * p.C, n = min(p.C, T - t0);
        if (col) {
            float* ckc = p.ck + ((size_t)bh * p.nch + c) * K * V;
#pragma unroll
            for (int i = 0; i < KMAX; ++i)
                if (i < K) ckc[(size_t)i * V + j] = S[i];
        }
        load_wv(t0, n);
        stage(t0, n, false);
#pragma unroll 1
        for (int r = 0; r < n; ++r) step(S, r, swv[r * nthr + j]);
    }

    // ---------------------------------------------------------------- pass 2: reverse
    float A[KMAX];
#pragma unroll
    for (int i = 0; i < KMAX; ++i) A[i] = (col && i < K && p.g_fin) ? p.g_fin[sbase + (size_t)i * V + j] : 0.f;
    int rb = 0;  // red[] buffer of the next reverse token
    for (int c = p.nch - 1; c >= 0; --c) {
        const int t0 = c * p.C, n = min(p.C, T - t0);
        // replay the chunk: previous states to the workspace, edits to registers
        const float* ckc = p.ck + ((size_t)bh * p.nch + c) * K * V;
#pragma unroll
        for (int i = 0; i < KMAX; ++i) S[i] = (col && i < K) ? ckc[(size_t)i * V + j] : 0.f;
        load_wv(t0, n);
        stage(t0, n, true);
#pragma unroll 1
        for (int r = 0; r < n; ++r) {
            float* rpr = p.rp + ((size_t)bh * p.C + r) * K * V;
            if (col) {
#pragma unroll
                for (int i = 0; i < KMAX; ++i)
                    if (i < K) rpr[(size_t)i * V + j] = S[i];
            }
            float x = step(S, r, swv[r * nthr + j]);
            x = col ? x : 0.f;
            sxe[r * nthr + j] = x;
            float x2 = x * x;
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) x2 += __shfl_xor_sync(FULL, x2, o);
            if (lane == 0) sen[r][warp] = x2;
        }
        __syncthreads();  // sen complete; the previous states are in the workspace (same thread)
        // walk the chunk backwards; the upstream gradient of the next token is fetched one step ahead
        float dy_next = (col && n > 0) ? p.g_out[tok(t0 + n - 1) * V + j] : 0.f;
#pragma unroll 1
        for (int r = n - 1; r >= 0; --r) {
            const int t = t0 + r;
            const size_t tk = tok(t) * K, tv = tok(t) * V;
            const float dy = dy_next;
            if (r > 0) dy_next = col ? p.g_out[tok(t - 1) * V + j] : 0.f;
            if (!sact[r]) {
                for (int x = j; x < K; x += nthr) p.dq[tk + x] = p.dk[tk + x] = p.dalpha[tk + x] = p.derase[tk + x] = 0.f;
                if (col) p.dv[tv + j] = p.dwrite[tv + j] = 0.f;
                continue;
            }
            const float wr = col ? p.write[tv + j] : 0.f, vr = col ? p.v[tv + j] : 0.f;
            const float* rpr = p.rp + ((size_t)bh * p.C + r) * K * V;
            float prev[KMAX];
#pragma unroll
            for (int i = 0; i < KMAX; ++i) prev[i] = (col && i < K) ? rpr[(size_t)i * V + j] : 0.f;
            const bool rst = srst[r];
            float en2 = 0.f;
            for (int w = 0; w < nwarps; ++w) en2 += sen[r][w];
            float kn2 = 0.f;
#pragma unroll
            for (int i = 0; i < KMAX; ++i) kn2 = fmaf(sk[r][i], sk[r][i], kn2);
            const float enorm = sqrtf(en2), knorm = sqrtf(kn2);
            const bool norms = knorm > 0.f && enorm > 0.f;
            const float gs = p.g_score ? p.g_score[tok(t)] : 0.f;
            const float key_scale = norms ? gs * enorm / knorm : 0.f;
            const float x_e = sxe[r * nthr + j];  // this column's edit (0 beyond V)
            float dd = (norms && col) ? gs * knorm * x_e / enorm : 0.f;
#pragma unroll
            for (int i = 0; i < KMAX; ++i) {
                A[i] = fmaf(sq[r][i], dy, A[i]);
                dd = fmaf(sk[r][i], A[i], dd);
            }
            if (!col) dd = 0.f;
            // the four per-channel sums, one 32-wide block at a time
#pragma unroll
            for (int kb = 0; kb < NKB; ++kb) {
                float vals[32];
#pragma unroll
                for (int u = 0; u < 32; ++u) {
                    const int i = 32 * kb + u;
                    const float bar = rst ? 0.f : sa[r][i] * prev[i];
                    vals[u] = (bar + sk[r][i] * x_e) * dy;
                }
                reduce_scatter32(vals, lane);
                red[rb][warp][0][32 * kb + lane] = vals[0];
#pragma unroll
                for (int u = 0; u < 32; ++u) {
                    const int i = 32 * kb + u;
                    const float bar = rst ? 0.f : sa[r][i] * prev[i];
                    vals[u] = A[i] * x_e - se[r][i] * bar * dd;
                }
                reduce_scatter32(vals, lane);
                red[rb][warp][1][32 * kb + lane] = vals[0];
#pragma unroll
                for (int u = 0; u < 32; ++u) {
                    const int i = 32 * kb + u;
                    const float bar = rst ? 0.f : sa[r][i] * prev[i];
                    vals[u] = -sk[r][i] * bar * dd;
                }
                reduce_scatter32(vals, lane);
                red[rb][warp][3][32 * kb + lane] = vals[0];
#pragma unroll
                for (int u = 0; u < 32; ++u) {
                    const int i = 32 * kb + u;
                    const float dbar = A[i] - se[r][i] * sk[r][i] * dd;
                    vals[u] = rst ? 0.f : dbar * prev[i];
                    A[i] = rst ? 0.f : sa[r][i] * dbar;
                }
                reduce_scatter32(vals, lane);
                red[rb][warp][2][32 * kb + lane] = vals[0];
            }
            if (col) {
                p.dv[tv + j] = dd * wr;
                p.dwrite[tv + j] = dd * vr;
            }
            __syncthreads();  // red[rb] complete; the other buffer takes the next token
            for (int x = j; x < 4 * K; x += nthr) {
                const int kind = x / K, i = x - kind * K;
                float s = 0.f;
                for (int w = 0; w < nwarps; ++w) s += red[rb][w][kind][i];
                if (kind == 0) p.dq[tk + i] = s;
                else if (kind == 1) p.dk[tk + i] = s + key_scale * sk[r][i];
                else if (kind == 2) p.dalpha[tk + i] = s;
                else p.derase[tk + i] = s;
            }
            rb ^= 1;
        }
    }
    if (p.dinitial && col) {
#pragma unroll
        for (int i = 0; i < KMAX; ++i)
            if (i < K) p.dinitial[sbase + (size_t)i * V + j] = A[i];

    }
}

int nchunks_of(int64_t T, int C) { return (int)((T + C - 1) / C); }

}  // namespace

size_t training_backward_workspace_bytes(int64_t B, int64_t T, int64_t H, int64_t K, int64_t V, int chunk) {
    if (B <= 0 || T <= 0 || H <= 0 || K <= 0 || V <= 0 || chunk < 1 || chunk > MAXC) return 0;
    const size_t heads = (size_t)B * H, kv = (size_t)K * V;
    return (heads * nchunks_of(T, chunk) * kv + heads * chunk * kv) * sizeof(float);
}

}  // namespace dbl

extern "C" size_t dbl_gdn_training_scan_backward_workspace_bytes(int64_t batch, int64_t time, int64_t heads,
                                                                 int64_t key_dim, int64_t value_dim,
                                                                 int32_t chunk_size) {
    return dbl::training_backward_workspace_bytes(batch, time, heads, key_dim, value_dim, chunk_size);
}

extern "C" int dbl_gdn_training_scan_backward(const dbl_training_scan_backward_args* a, void* workspace,
                                              size_t workspace_bytes, dbl_stream_t stream) {
    using namespace dbl;
    if (!a) return fail(DBL_ERR_INVALID_ARGUMENT, "gdn_training_scan_backward: null args");
    if (a->batch <= 0 || a->time <= 0 || a->heads <= 0 || a->key_dim <= 0 || a->value_dim <= 0)
        return fail(DBL_ERR_INVALID_ARGUMENT, "GDN-2 requires nonempty axes");
    if (a->chunk_size < 1 || a->chunk_size > MAXC)
        return fail(DBL_ERR_INVALID_ARGUMENT, "GDN-2 checkpoint chunk must be 1..=16");
    if (!a->q || !a->k || !a->v || !a->alpha || !a->erase || !a->write || !a->valid || !a->reset || !a->grad_output ||
        !a->dq || !a->dk || !a->dv || !a->dalpha || !a->derase || !a->dwrite)
        return fail(DBL_ERR_INVALID_ARGUMENT,
                    "gdn_training_scan_backward: q, k, v, alpha, erase, write, valid, reset, grad_output and the "
                    "six input gradients are required");
    if (a->key_dim > 64 || a->value_dim > 256)
        return fail(DBL_ERR_UNSUPPORTED, "gdn_training_scan_backward: key width up to 64 and value width up to 256");
    if (a->batch * a->heads > 0x7fffffff || a->time > 0x7fffffff)
        return fail(DBL_ERR_UNSUPPORTED, "GDN-2 axis exceeds 32-bit limits");
    const size_t need = training_backward_workspace_bytes(a->batch, a->time, a->heads, a->key_dim, a->value_dim,
                                                          a->chunk_size);
    if (!workspace || workspace_bytes < need)
        return fail(DBL_ERR_WORKSPACE, "gdn_training_scan_backward: workspace of %zu bytes required (got %zu)", need,
                    workspace_bytes);
    BwdParams p{};
    p.B = (int)a->batch;
    p.T = (int)a->time;
    p.H = (int)a->heads;
    p.K = (int)a->key_dim;
    p.V = (int)a->value_dim;
    p.C = a->chunk_size;
    p.nch = nchunks_of(a->time, a->chunk_size);
    p.q = a->q;
    p.k = a->k;
    p.v = a->v;
    p.alpha = a->alpha;
    p.erase = a->erase;
    p.write = a->write;
    p.valid = a->valid;
    p.reset = a->reset;
    p.initial = a->initial_state;
    p.g_out = a->grad_output;
    p.g_fin = a->grad_final_state;
    p.g_score = a->grad_scores;
    p.dq = a->dq;
    p.dk = a->dk;
    p.dv = a->dv;
    p.dalpha = a->dalpha;
    p.derase = a->derase;
    p.dwrite = a->dwrite;
    p.dinitial = a->dinitial;
    const size_t heads = (size_t)a->batch * a->heads;
    p.ck = static_cast<float*>(workspace);
    p.rp = p.ck + heads * p.nch * (size_t)p.K * p.V;
    const int threads = (p.V + 31) / 32 * 32;
    const size_t dyn = 2 * (size_t)MAXC * threads * sizeof(float);  // swv, sxe
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    static std::atomic<uint64_t> attr_done{0};  // the dynamic part may take the static part past 48 KB
    const int rc = once_per_device(attr_done, [] {
        cudaError_t e = cudaFuncSetAttribute(training_backward_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             2 * MAXC * 256 * (int)sizeof(float));
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(training_backward_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     2 * MAXC * 256 * (int)sizeof(float));
        return cuda_status(e, "gdn_training_scan_backward: cudaFuncSetAttribute");
    });
    if (rc != DBL_OK) return rc;
    if (p.K <= 32) training_backward_kernel<32><<<(unsigned)heads, threads, dyn, st>>>(p);
    else training_backward_kernel<64><<<(unsigned)heads, threads, dyn, st>>>(p);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? DBL_OK : cuda_status(e, "gdn_training_scan_backward launch");
}

// ------------------------------------------------------------------------------ gdn2_scan backward
// The output-only scan with inclusive document limits (dbl_gdn2_scan) is the stateful scan with
// valid = (doc_end >= doc_start), reset = (doc_start == t), a zero initial state and no final state
// or scores, so its backward (gdn2_backward, crates/kernels/src/gdn2.rs:285-519, wired at
// ops.rs:106-160) is the kernel above on those masks, with zero final-state and score gradients.
namespace dbl {
namespace {

__global__ void limits_to_masks_kernel(const int32_t* start, const int32_t* end, int64_t B, int64_t T, float* valid,
                                       float* reset) {
    const int64_t x = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (x >= B * T) return;
    const int t = (int)(x % T);
    valid[x] = end[x] >= start[x] ? 1.f : 0.f;
    reset[x] = start[x] == t ? 1.f : 0.f;
}
__global__ void widen_bf16_kernel(const __nv_bfloat16* in, float* out, int64_t n) {
    for (int64_t x = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; x < n; x += (int64_t)gridDim.x * blockDim.x)
        out[x] = __bfloat162float(in[x]);
}
__global__ void narrow_bf16_kernel(const float* in, __nv_bfloat16* out, int64_t n) {
    for (int64_t x = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; x < n; x += (int64_t)gridDim.x * blockDim.x)
        out[x] = __float2bfloat16_rn(in[x]);
}

constexpr int GDN2_CHUNK = 16;  // gdn2.rs: C = 16
size_t al256(size_t x) { return (x + 255) & ~size_t(255); }

struct Gdn2BwdLayout {
    size_t valid, reset, q, k, v, go, dq, dk, dv, train, total;
};
Gdn2BwdLayout gdn2_bwd_layout(int64_t B, int64_t T, int64_t H, int64_t K, int64_t V, int dtype) {
    Gdn2BwdLayout L{};
    const size_t bt = (size_t)(B * T), nk = (size_t)(B * T * H * K) * 4, nv = (size_t)(B * T * H * V) * 4;
    const bool wide = dtype == DBL_BF16;
    size_t o = 0;
    L.valid = o; o += al256(bt * 4);
    L.reset = o; o += al256(bt * 4);
    L.q = o; o += wide ? al256(nk) : 0;
    L.k = o; o += wide ? al256(nk) : 0;
    L.v = o; o += wide ? al256(nv) : 0;
    L.go = o; o += wide ? al256(nv) : 0;
    L.dq = o; o += wide ? al256(nk) : 0;
    L.dk = o; o += wide ? al256(nk) : 0;
    L.dv = o; o += wide ? al256(nv) : 0;
    L.train = o; o += training_backward_workspace_bytes(B, T, H, K, V, GDN2_CHUNK);
    L.total = o;
    return L;
}

unsigned grid_for(int64_t n) { return (unsigned)std::min<int64_t>((n + 255) / 256, 148 * 16); }

}  // namespace
}  // namespace dbl

extern "C" size_t dbl_gdn2_scan_backward_workspace_bytes(int64_t batch, int64_t time, int64_t heads, int64_t key_dim,
                                                         int64_t value_dim, int32_t dtype) {
    if (batch <= 0 || time <= 0 || heads <= 0 || key_dim <= 0 || value_dim <= 0) return 0;
    return dbl::gdn2_bwd_layout(batch, time, heads, key_dim, value_dim, dtype).total;
}

extern "C" int dbl_gdn2_scan_backward(const dbl_gdn2_scan_backward_args* a, void* workspace, size_t workspace_bytes,
                                      dbl_stream_t stream) {
    using namespace dbl;
    if (!a) return fail(DBL_ERR_INVALID_ARGUMENT, "gdn2_scan_backward: null args");
    if (a->batch <= 0 || a->time <= 0 || a->heads <= 0 || a->key_dim <= 0 || a->value_dim <= 0)
        return fail(DBL_ERR_INVALID_ARGUMENT, "GDN-2 requires nonempty axes");
    if (a->dtype != DBL_F32 && a->dtype != DBL_BF16)
        return fail(DBL_ERR_INVALID_ARGUMENT, "gdn2_scan_backward: dtype must be f32 or bf16");
    if (!a->q || !a->k || !a->v || !a->alpha || !a->erase || !a->write || !a->doc_start || !a->doc_end ||
        !a->grad_output || !a->dq || !a->dk || !a->dv || !a->dalpha || !a->derase || !a->dwrite)
        return fail(DBL_ERR_INVALID_ARGUMENT, "gdn2_scan_backward: every pointer is required");
    const Gdn2BwdLayout L = gdn2_bwd_layout(a->batch, a->time, a->heads, a->key_dim, a->value_dim, a->dtype);
    if (!workspace || workspace_bytes < L.total)
        return fail(DBL_ERR_WORKSPACE, "gdn2_scan_backward: workspace of %zu bytes required (got %zu)", L.total,
                    workspace_bytes);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    const int64_t bt = a->batch * a->time, nk = bt * a->heads * a->key_dim, nv = bt * a->heads * a->value_dim;
    float* valid = reinterpret_cast<float*>(ws + L.valid);
    float* reset = reinterpret_cast<float*>(ws + L.reset);
    limits_to_masks_kernel<<<(unsigned)((bt + 255) / 256), 256, 0, st>>>(a->doc_start, a->doc_end, a->batch, a->time,
                                                                         valid, reset);
    const bool wide = a->dtype == DBL_BF16;
    dbl_training_scan_backward_args t{};
    t.batch = a->batch;
    t.time = a->time;
    t.heads = a->heads;
    t.key_dim = a->key_dim;
    t.value_dim = a->value_dim;
    t.chunk_size = GDN2_CHUNK;
    if (wide) {
        float *q = reinterpret_cast<float*>(ws + L.q), *k = reinterpret_cast<float*>(ws + L.k);
        float *v = reinterpret_cast<float*>(ws + L.v), *go = reinterpret_cast<float*>(ws + L.go);
        widen_bf16_kernel<<<grid_for(nk), 256, 0, st>>>(static_cast<const __nv_bfloat16*>(a->q), q, nk);
        widen_bf16_kernel<<<grid_for(nk), 256, 0, st>>>(static_cast<const __nv_bfloat16*>(a->k), k, nk);
        widen_bf16_kernel<<<grid_for(nv), 256, 0, st>>>(static_cast<const __nv_bfloat16*>(a->v), v, nv);
        widen_bf16_kernel<<<grid_for(nv), 256, 0, st>>>(static_cast<const __nv_bfloat16*>(a->grad_output), go, nv);
        t.q = q;
        t.k = k;
        t.v = v;
        t.grad_output = go;
        t.dq = reinterpret_cast<float*>(ws + L.dq);
        t.dk = reinterpret_cast<float*>(ws + L.dk);
        t.dv = reinterpret_cast<float*>(ws + L.dv);
    } else {
        t.q = static_cast<const float*>(a->q);
        t.k = static_cast<const float*>(a->k);
        t.v = static_cast<const float*>(a->v);
        t.grad_output = static_cast<const float*>(a->grad_output);
        t.dq = static_cast<float*>(a->dq);
        t.dk = static_cast<float*>(a->dk);
        t.dv = static_cast<float*>(a->dv);
    }
    t.alpha = a->alpha;
    t.erase = a->erase;
    t.write = a->write;
    t.valid = valid;
    t.reset = reset;
    t.dalpha = a->dalpha;
    t.derase = a->derase;
    t.dwrite = a->dwrite;
    const int rc = dbl_gdn_training_scan_backward(&t, ws + L.train, L.total - L.train, stream);
    if (rc != DBL_OK) return rc;
    if (wide) {
        narrow_bf16_kernel<<<grid_for(nk), 256, 0, st>>>(t.dq, static_cast<__nv_bfloat16*>(a->dq), nk);
        narrow_bf16_kernel<<<grid_for(nk), 256, 0, st>>>(t.dk, static_cast<__nv_bfloat16*>(a->dk), nk);
        narrow_bf16_kernel<<<grid_for(nv), 256, 0, st>>>(t.dv, static_cast<__nv_bfloat16*>(a->dv), nv);
    }
    return launch_status("gdn2_scan_backward");
}
