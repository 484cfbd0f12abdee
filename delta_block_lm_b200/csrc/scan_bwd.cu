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
#include "scan_seq_params.cuh"

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
    int rp_shared;  // 1: those states live in shared memory ([C][K][cols + 8]) instead of rp
};

// One level of a reduce-scatter over the lanes that differ in lane bit `o`: the lower lane keeps
// (and sums) the first `half` values, the upper lane the next `half`, moved to the front.
template <int N>
__device__ __forceinline__ void rs_level(float (&v)[N], int half, int o, int lane) {
    const bool upper = (lane & o) != 0;
#pragma unroll
    for (int x = 0; x < N / 2; ++x) {
        if (x < half) {
            const float send = upper ? v[x] : v[x + half];
            const float keep = upper ? v[x + half] : v[x];
            v[x] = keep + __shfl_xor_sync(FULL, send, o);
        }
    }
}
// Sums v over the 32 / TPC lanes that share lane % TPC (the columns of the warp at one row group):
// afterwards v[0 .. M), M = N TPC / 32, holds the sums of indices [M s, M (s + 1)), s = lane / TPC.
template <int N, int TPC>
__device__ __forceinline__ void reduce_scatter_cols(float (&v)[N], int lane) {
    int half = N / 2;
#pragma unroll
    for (int o = 16; o >= TPC; o >>= 1) {
        rs_level(v, half, o, lane);
        half >>= 1;
    }
}
template <int TPC>
__device__ __forceinline__ float row_sum(float x) {
#pragma unroll
    for (int o = 1; o < TPC; o <<= 1) x += __shfl_xor_sync(FULL, x, o);
    return x;
}

// Shared memory of the backward kernel (dynamic; the same carve-up on host and device).
struct BwdSmem {
    size_t k, a, e, q, wv, xe, en, kn, gs, red, act, rst, total;
};
__host__ __device__ inline BwdSmem bwd_smem(int kmax, int cols, int nwarps) {
    BwdSmem L{};
    size_t o = 0;
    const size_t tk = (size_t)MAXC * kmax * 4, tc = (size_t)MAXC * cols * 4;
    L.k = o; o += tk;
    L.a = o; o += tk;
    L.e = o; o += tk;
    L.q = o; o += tk;
    L.wv = o; o += tc;
    L.xe = o; o += tc;
    L.en = o; o += MAXC * 4;
    L.kn = o; o += MAXC * 4;
    L.gs = o; o += MAXC * 4;
    L.red = o; o += (size_t)2 * nwarps * 4 * kmax * 4;
    L.act = o; o += MAXC * 4;
    L.rst = o; o += MAXC * 4;
    L.total = o;
    return L;
}

// TPC lanes share value column j (as the forward kernel): lane g = lane % TPC holds state, adjoint
// and replayed rows i = g, g + TPC, ... (R = KMAX / TPC of them).
template <int KMAX, int TPC>
__global__ void __launch_bounds__(512) training_backward_kernel(const BwdParams p) {
    constexpr int R = KMAX / TPC;
    constexpr int NV = 4 * R;            // per-lane contributions to the four channel sums
    constexpr int M = NV * TPC / 32;     // sums a lane holds after the column reduce-scatter
    extern __shared__ __align__(16) uint8_t dyn_raw[];
    const int tid = threadIdx.x, nthr = blockDim.x;
    const int warp = tid >> 5, lane = tid & 31, nwarps = nthr >> 5;
    const int g = lane % TPC;
    const int j = warp * (32 / TPC) + lane / TPC;  // value column
    const int cols = nwarps * (32 / TPC);
    const BwdSmem L = bwd_smem(KMAX, cols, nwarps);
    float(*sk)[KMAX] = reinterpret_cast<float(*)[KMAX]>(dyn_raw + L.k);
    float(*sa)[KMAX] = reinterpret_cast<float(*)[KMAX]>(dyn_raw + L.a);
    float(*se)[KMAX] = reinterpret_cast<float(*)[KMAX]>(dyn_raw + L.e);
    float(*sq)[KMAX] = reinterpret_cast<float(*)[KMAX]>(dyn_raw + L.q);
    float* swv = reinterpret_cast<float*>(dyn_raw + L.wv);  // [MAXC][cols]
    float* sxe = reinterpret_cast<float*>(dyn_raw + L.xe);  // [MAXC][cols]
    float* sen = reinterpret_cast<float*>(dyn_raw + L.en);  // |edit|^2 per token
    float* skn = reinterpret_cast<float*>(dyn_raw + L.kn);  // |k|^2 per token
    float* sgs = reinterpret_cast<float*>(dyn_raw + L.gs);  // g_score per token
    float* red = reinterpret_cast<float*>(dyn_raw + L.red); // [2][nwarps][4][KMAX]
    int* sact = reinterpret_cast<int*>(dyn_raw + L.act);
    int* srst = reinterpret_cast<int*>(dyn_raw + L.rst);
    // the replayed previous states of the chunk: shared memory when they fit (row stride cols + 8
    // puts the four row-group lanes of a column on different banks), else this CTA's workspace rows
    const int rstride = p.rp_shared ? cols + 8 : p.V;
    float* rpb = p.rp_shared ? reinterpret_cast<float*>(dyn_raw + L.total)
                             : p.rp + (size_t)blockIdx.x * p.C * p.K * p.V;

    const int bh = blockIdx.x;
    const int b = bh / p.H, h = bh - b * p.H;
    const bool col = j < p.V;
    const int K = p.K, V = p.V, T = p.T, H = p.H;
    const size_t sbase = ((size_t)b * H + h) * K * V;
    auto tok = [&](int t) { return ((size_t)b * T + t) * H + h; };  // token row index

    // stages the n tokens from t0 (k, alpha, erase and, for the reverse, q) with one pair of
    // barriers: every load of the chunk is in flight at once
    auto stage = [&](int t0, int n, bool with_q) {
        __syncthreads();
        for (int x = tid; x < n * KMAX; x += nthr) {
            const int r = x / KMAX, i = x - r * KMAX;
            const bool in = i < K;
            const size_t gi = tok(t0 + r) * K + i;
            sk[r][i] = in ? p.k[gi] : 0.f;
            sa[r][i] = in ? p.alpha[gi] : 0.f;
            se[r][i] = in ? p.erase[gi] : 0.f;
            if (with_q) sq[r][i] = in ? p.q[gi] : 0.f;
        }
        if (tid < n) {
            sact[tid] = p.valid[(size_t)b * T + t0 + tid] != 0.f;
            srst[tid] = p.reset[(size_t)b * T + t0 + tid] != 0.f;
            if (with_q) sgs[tid] = p.g_score ? p.g_score[tok(t0 + tid)] : 0.f;
        }
        if (g == 0) {
            // this column's write * v for the chunk: all loads issued, then stored
            float w[MAXC], x[MAXC];
#pragma unroll
            for (int r = 0; r < MAXC; ++r) {
                w[r] = (col && r < n) ? p.write[tok(t0 + r) * V + j] : 0.f;
                x[r] = (col && r < n) ? p.v[tok(t0 + r) * V + j] : 0.f;
            }
#pragma unroll
            for (int r = 0; r < MAXC; ++r) swv[r * cols + j] = w[r] * x[r];
        }
        __syncthreads();
    };
    // one forward step of this lane's rows; returns the column's edit x
    auto step = [&](float (&S)[R], int r) {
        if (!sact[r]) return 0.f;
        const bool rst = srst[r];
        float part = 0.f;
#pragma unroll
        for (int u = 0; u < R; ++u) {
            const int i = g + TPC * u;
            const float bar = rst ? 0.f : sa[r][i] * S[u];
            part = fmaf(se[r][i] * sk[r][i], bar, part);
            S[u] = bar;
        }
        const float x = (col ? swv[r * cols + j] : 0.f) - row_sum<TPC>(part);
#pragma unroll
        for (int u = 0; u < R; ++u) S[u] = fmaf(sk[r][g + TPC * u], x, S[u]);
        return x;
    };
    auto row_ok = [&](int u) { return col && g + TPC * u < K; };

    // ---------------------------------------------------------------- pass 1: checkpoints
    float S[R];
#pragma unroll
    for (int u = 0; u < R; ++u) S[u] = (row_ok(u) && p.initial) ? p.initial[sbase + (size_t)(g + TPC * u) * V + j] : 0.f;
    for (int c = 0; c < p.nch; ++c) {
        const int t0 = c * p.C, n = min(p.C, T - t0);
        float* ckc = p.ck + ((size_t)bh * p.nch + c) * K * V;
#pragma unroll
        for (int u = 0; u < R; ++u)
            if (row_ok(u)) ckc[(size_t)(g + TPC * u) * V + j] = S[u];
        stage(t0, n, false);
#pragma unroll 1
        for (int r = 0; r < n; ++r) step(S, r);
    }

    // ---------------------------------------------------------------- pass 2: reverse
    float A[R];
#pragma unroll
    for (int u = 0; u < R; ++u) A[u] = (row_ok(u) && p.g_fin) ? p.g_fin[sbase + (size_t)(g + TPC * u) * V + j] : 0.f;
    int rb = 0;  // red buffer of the next reverse token
    for (int c = p.nch - 1; c >= 0; --c) {
        const int t0 = c * p.C, n = min(p.C, T - t0);
        // replay the chunk: previous states to the workspace, edits to shared memory
        const float* ckc = p.ck + ((size_t)bh * p.nch + c) * K * V;
#pragma unroll
        for (int u = 0; u < R; ++u) S[u] = row_ok(u) ? ckc[(size_t)(g + TPC * u) * V + j] : 0.f;
        stage(t0, n, true);
#pragma unroll 1
        for (int r = 0; r < n; ++r) {
            float* rpr = rpb + (size_t)r * K * rstride;
#pragma unroll
            for (int u = 0; u < R; ++u)
                if (row_ok(u)) rpr[(size_t)(g + TPC * u) * rstride + j] = S[u];
            const float x = step(S, r);
            if (g == 0 && col) sxe[r * cols + j] = x;
        }
        __syncthreads();
        // |edit|^2 and |k|^2 of each token of the chunk: one warp per token
        for (int r = warp; r < n; r += nwarps) {
            float e2 = 0.f, k2 = 0.f;
            for (int cc = lane; cc < V; cc += 32) e2 = fmaf(sxe[r * cols + cc], sxe[r * cols + cc], e2);
            for (int i = lane; i < K; i += 32) k2 = fmaf(sk[r][i], sk[r][i], k2);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                e2 += __shfl_xor_sync(FULL, e2, o);
                k2 += __shfl_xor_sync(FULL, k2, o);
            }
            if (lane == 0) {
                sen[r] = e2;
                skn[r] = k2;
            }
        }
        __syncthreads();
        // walk the chunk backwards; the upstream gradient of the next token is fetched one step ahead
        float dy_next = (col && n > 0) ? p.g_out[tok(t0 + n - 1) * V + j] : 0.f;
#pragma unroll 1
        for (int r = n - 1; r >= 0; --r) {
            const int t = t0 + r;
            const size_t tk = tok(t) * K, tv = tok(t) * V;
            const float dy = dy_next;
            if (r > 0) dy_next = col ? p.g_out[tok(t - 1) * V + j] : 0.f;
            if (!sact[r]) {
                for (int x = tid; x < K; x += nthr) p.dq[tk + x] = p.dk[tk + x] = p.dalpha[tk + x] = p.derase[tk + x] = 0.f;
                if (col && g == 0) p.dv[tv + j] = p.dwrite[tv + j] = 0.f;
                continue;
            }
            const float wr = (col && g == 0) ? p.write[tv + j] : 0.f, vr = (col && g == 0) ? p.v[tv + j] : 0.f;
            const float* rpr = rpb + (size_t)r * K * rstride;
            float prev[R];
#pragma unroll
            for (int u = 0; u < R; ++u) prev[u] = row_ok(u) ? rpr[(size_t)(g + TPC * u) * rstride + j] : 0.f;
            const bool rst = srst[r];
            const float enorm = sqrtf(sen[r]), knorm = sqrtf(skn[r]);
            const bool norms = knorm > 0.f && enorm > 0.f;
            const float gs = sgs[r];
            const float key_scale = norms ? gs * enorm / knorm : 0.f;
            const float x_e = col ? sxe[r * cols + j] : 0.f;  // this column's edit
            float part = 0.f;
#pragma unroll
            for (int u = 0; u < R; ++u) {
                const int i = g + TPC * u;
                A[u] = fmaf(sq[r][i], dy, A[u]);
                part = fmaf(sk[r][i], A[u], part);
            }
            float dd = row_sum<TPC>(part) + ((norms && col) ? gs * knorm * x_e / enorm : 0.f);
            if (!col) dd = 0.f;
            // the four per-channel contributions of this lane's rows: [q][u], q = dq, dk, dalpha, derase
            float vals[NV];
#pragma unroll
            for (int u = 0; u < R; ++u) {
                const int i = g + TPC * u;
                const float bar = rst ? 0.f : sa[r][i] * prev[u];
                const float dbar = A[u] - se[r][i] * sk[r][i] * dd;
                vals[u] = (bar + sk[r][i] * x_e) * dy;
                vals[R + u] = A[u] * x_e - se[r][i] * bar * dd;
                vals[2 * R + u] = rst ? 0.f : dbar * prev[u];
                vals[3 * R + u] = -sk[r][i] * bar * dd;
                A[u] = rst ? 0.f : sa[r][i] * dbar;
            }
            reduce_scatter_cols<NV, TPC>(vals, lane);
            {
                const int s = lane / TPC;
                float* rw = red + ((size_t)(rb * nwarps + warp) * 4) * KMAX;
#pragma unroll
                for (int m = 0; m < M; ++m) {
                    const int idx = M * s + m, q = idx / R, u = idx - q * R;
                    rw[q * KMAX + g + TPC * u] = vals[m];
                }
            }
            if (col && g == 0) {
                p.dv[tv + j] = dd * wr;
                p.dwrite[tv + j] = dd * vr;
            }
            __syncthreads();  // red[rb] complete; the other buffer takes the next token
            for (int x = tid; x < 4 * K; x += nthr) {
                const int q = x / K, i = x - q * K;
                float sum = 0.f;
                for (int w = 0; w < nwarps; ++w) sum += red[((size_t)(rb * nwarps + w) * 4 + q) * KMAX + i];
                if (q == 0) p.dq[tk + i] = sum;
                else if (q == 1) p.dk[tk + i] = sum + key_scale * sk[r][i];
                else if (q == 2) p.dalpha[tk + i] = sum;
                else p.derase[tk + i] = sum;
            }
            rb ^= 1;
        }
    }
    if (p.dinitial) {
#pragma unroll
        for (int u = 0; u < R; ++u)
            if (row_ok(u)) p.dinitial[sbase + (size_t)(g + TPC * u) * V + j] = A[u];
    }
}

int nchunks_of(int64_t T, int C) { return (int)((T + C - 1) / C); }

}  // namespace

// Whether the backward of these shapes runs in the chunked form (scan_chunk_bwd.cu): 16-token
// checkpoints and the shapes chunk_backward_supported takes.
bool chunked_backward(int64_t B, int64_t T, int64_t H, int64_t K, int64_t V, int chunk) {
    if (chunk != 16 || B > 0x7fffffff || T > 0x7fffffff || H > 0x7fffffff || K > 64 || V > 256) return false;
    const SeqParams sp = chunk_backward_forward_params((int)B, (int)T, (int)H, (int)K, (int)V, nullptr, nullptr,
                                                       nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr);
    return chunk_backward_supported(sp);
}

size_t training_backward_workspace_bytes(int64_t B, int64_t T, int64_t H, int64_t K, int64_t V, int chunk) {
    if (B <= 0 || T <= 0 || H <= 0 || K <= 0 || V <= 0 || chunk < 1 || chunk > MAXC) return 0;
    const size_t heads = (size_t)B * H, kv = (size_t)K * V;
    size_t bytes = (heads * nchunks_of(T, chunk) * kv + heads * chunk * kv) * sizeof(float);
    if (chunked_backward(B, T, H, K, V, chunk)) {
        const SeqParams sp = chunk_backward_forward_params((int)B, (int)T, (int)H, (int)K, (int)V, nullptr, nullptr,
                                                           nullptr, nullptr, nullptr, nullptr, nullptr, nullptr,
                                                           nullptr);
        bytes = std::max(bytes, chunk_backward_workspace_floats(sp) * sizeof(float));
    }
    return bytes;
}

}  // namespace dbl

extern "C" size_t dbl_gdn_training_scan_backward_workspace_bytes(int64_t batch, int64_t time, int64_t heads,
                                                                 int64_t key_dim, int64_t value_dim,
                                                                 int32_t chunk_size) {
    return dbl::training_backward_workspace_bytes(batch, time, heads, key_dim, value_dim, chunk_size);
}

namespace dbl {

// The backward entry, recomputing the forward (ctx null) or reading a saved context at the shapes
// that keep one (chunked_backward).
int training_backward_entry(const dbl_training_scan_backward_args* a, void* workspace, size_t workspace_bytes,
                            const void* ctx, size_t ctx_bytes, dbl_stream_t stream) {
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
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    // 16-token checkpoints at the shapes of the chunked forward: the chunked backward
    // (scan_chunk_bwd.cu), given a 16-byte aligned workspace
    const bool chunked = chunked_backward(a->batch, a->time, a->heads, a->key_dim, a->value_dim, a->chunk_size);
    if (chunked && ctx) {
        // the saved context of dbl_gdn_training_scan_save (16-byte aligned, checked by the caller)
        const SeqParams sp = chunk_backward_forward_params(p.B, p.T, p.H, p.K, p.V, p.q, p.k, p.v, p.alpha, p.erase,
                                                           p.write, p.valid, p.reset, p.initial);
        if (ctx_bytes < chunk_context_floats(sp) * sizeof(float))
            return fail(DBL_ERR_WORKSPACE, "gdn_training_scan_backward_saved: context of %zu bytes required (got %zu)",
                        chunk_context_floats(sp) * sizeof(float), ctx_bytes);
        if ((reinterpret_cast<uintptr_t>(workspace) & 15) != 0)
            return fail(DBL_ERR_INVALID_ARGUMENT, "gdn_training_scan_backward_saved: workspace must be 16-byte aligned");
        return launch_chunk_backward_saved(sp, p.g_out, p.g_fin, p.g_score, p.dq, p.dk, p.dv, p.dalpha, p.derase,
                                           p.dwrite, p.dinitial, static_cast<const float*>(ctx),
                                           static_cast<float*>(workspace), st);
    }
    if (chunked && (reinterpret_cast<uintptr_t>(workspace) & 15) == 0) {
        const SeqParams sp = chunk_backward_forward_params(p.B, p.T, p.H, p.K, p.V, p.q, p.k, p.v, p.alpha, p.erase,
                                                           p.write, p.valid, p.reset, p.initial);
        return launch_chunk_backward(sp, p.g_out, p.g_fin, p.g_score, p.dq, p.dk, p.dv, p.dalpha, p.derase, p.dwrite,
                                     p.dinitial, static_cast<float*>(workspace), st);
    }
    // four lanes per value column up to 128 columns, two beyond (at most 512 threads)
    const int tpc = p.V <= 128 ? 4 : 2;
    const int threads = (p.V * tpc + 31) / 32 * 32, nwarps = threads / 32;
    const int cols = nwarps * (32 / tpc);
    const size_t base_smem = bwd_smem(p.K <= 32 ? 32 : 64, cols, nwarps).total;
    const size_t rp_smem = (size_t)p.C * p.K * (cols + 8) * sizeof(float);
    p.rp_shared = base_smem + rp_smem <= 200 * 1024 ? 1 : 0;  // a chunk's replayed states fit on chip
    const size_t dyn = base_smem + (p.rp_shared ? rp_smem : 0);
    auto go = [&](auto kernel) {
        if (dyn > 48 * 1024) {
            const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dyn);
            if (e != cudaSuccess) return e;
        }
        kernel<<<(unsigned)heads, threads, dyn, st>>>(p);
        return cudaGetLastError();
    };
    cudaError_t e;
    if (p.K <= 32) e = tpc == 4 ? go(training_backward_kernel<32, 4>) : go(training_backward_kernel<32, 2>);
    else e = tpc == 4 ? go(training_backward_kernel<64, 4>) : go(training_backward_kernel<64, 2>);
    return e == cudaSuccess ? DBL_OK : cuda_status(e, "gdn_training_scan_backward launch");
}

}  // namespace dbl

extern "C" int dbl_gdn_training_scan_backward(const dbl_training_scan_backward_args* a, void* workspace,
                                              size_t workspace_bytes, dbl_stream_t stream) {
    return dbl::training_backward_entry(a, workspace, workspace_bytes, nullptr, 0, stream);
}

// The reference's forward returns checkpoint and auxiliary tensors beside its outputs and its
// backward consumes them (gdn_training_ops.rs:201-224, :87-112).  These three calls do the same:
// at the shapes of the chunked backward the context holds the chunk-start states, the chunk maps and
// every token's edit; elsewhere it is empty (0 bytes) and the two calls are the plain forward and the
// recomputing backward.
extern "C" size_t dbl_gdn_training_scan_context_bytes(int64_t batch, int64_t time, int64_t heads, int64_t key_dim,
                                                      int64_t value_dim, int32_t chunk_size) {
    using namespace dbl;
    if (batch <= 0 || time <= 0 || heads <= 0 || key_dim <= 0 || value_dim <= 0 || chunk_size < 1 ||
        chunk_size > MAXC)
        return 0;
    if (!chunked_backward(batch, time, heads, key_dim, value_dim, chunk_size)) return 0;
    const SeqParams sp = chunk_backward_forward_params((int)batch, (int)time, (int)heads, (int)key_dim, (int)value_dim,
                                                       nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr,
                                                       nullptr, nullptr);
    return chunk_context_floats(sp) * sizeof(float);
}

extern "C" int dbl_gdn_training_scan_save(const dbl_training_scan_args* a, void* context, size_t context_bytes,
                                          dbl_stream_t stream) {
    using namespace dbl;
    SeqParams p{};
    int rc = training_scan_params(a, &p);
    if (rc != DBL_OK) return rc;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const size_t need =
        dbl_gdn_training_scan_context_bytes(a->batch, a->time, a->heads, a->key_dim, a->value_dim, a->chunk_size);
    if (need == 0) return launch_seq_scan(p, a->dtype, st);
    if (!context || context_bytes < need)
        return fail(DBL_ERR_WORKSPACE, "gdn_training_scan_save: context of %zu bytes required (got %zu)", need,
                    context_bytes);
    if ((reinterpret_cast<uintptr_t>(context) & 15) != 0)
        return fail(DBL_ERR_INVALID_ARGUMENT, "gdn_training_scan_save: context must be 16-byte aligned");
    return launch_chunk_forward_saved(p, a->dtype, static_cast<float*>(context), st);
}

extern "C" int dbl_gdn_training_scan_backward_saved(const dbl_training_scan_backward_args* a, const void* context,
                                                    size_t context_bytes, void* workspace, size_t workspace_bytes,
                                                    dbl_stream_t stream) {
    using namespace dbl;
    if (a && context && (reinterpret_cast<uintptr_t>(context) & 15) != 0)
        return fail(DBL_ERR_INVALID_ARGUMENT, "gdn_training_scan_backward_saved: context must be 16-byte aligned");
    if (a && !context &&
        dbl_gdn_training_scan_context_bytes(a->batch, a->time, a->heads, a->key_dim, a->value_dim, a->chunk_size) > 0)
        return fail(DBL_ERR_WORKSPACE, "gdn_training_scan_backward_saved: these shapes keep a context; pass it");
    return training_backward_entry(a, workspace, workspace_bytes, context, context_bytes, stream);
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
