// Long-sequence prefill by time segments: the span-map fold, the one-device
// segmented prefill and the multi-device time-sharded prefill driven from one host thread.
//
// Over a token span the GDN-2 state map is affine: S_end = A S_start + B, with A the K x K span
// transition (dbl_gdn2_span_transition: the scan of the span from S = I with zero values) and B
// the scan of the span from a zero state.  A span of T tokens is cut into `segments` equal
// segments that run as a batch (a strided [segments, T/segments, H, D] view of the same memory),
// so segments x H CTAs of the tensor-core prefill share the GPU instead of H:
//   pass 1  the maps (A_s, B_s) of every segment (two batched launches);
//   fold    the start state of every segment, X_{s+1} = A_s X_s + B_s (span_fold_kernel);
//   pass 2  every segment rescanned from its start state (one batched launch).
// On one device the default schedule (segments = 0, lead_prefill) cuts the span into a lead
// segment and m = SMs / H equal segments instead: the lead needs no maps, so it is scanned from the
// initial state on a side stream while pass 1 runs over segments 1 .. m-1 (the last segment needs
// no maps either), and the fold and one rescan of segments 1 .. m follow.
// Across devices, device g holds time span g.  Each device composes its span's map
// (A_g, B_g) = fold of its segment maps; device 0 instead folds its maps from the sequence's initial
// state to its end state E_0.  Device g pulls E_0 and the maps of devices 1 .. g-1 with one
// cudaMemcpyPeerAsync each (ordered after the producing device's event), folds them into its start
// state and runs its own fold and pass 2.  Peer memory is only read by copies, never by a kernel.
// The reference has no time-parallel or multi-device code; this file is the B200 build's own.
#include <mutex>
#include <vector>

#include "common.cuh"
#include "tc_ptx.cuh"

namespace dbl {

int prefill_dispatch(const dbl_prefill_args* a, int mode, float* transition, cudaStream_t st);

namespace {

constexpr int kFoldLdA = 132;  // row stride (floats) of a staged transition: 8 rows read at one k hit distinct banks
constexpr int kFoldStages = 2;  // transitions in flight: A_{s+1} loads while step s computes
constexpr int kChunk = 64;

// One fold: X_{s+1} = A_s X_s + B_s over `V` columns.
struct FoldJob {
    int V;
    const float* B;    // [S][H][K][V] or null (zero offsets)
    const float* X0;   // [H][K][V] or null (zeros); ignored when x0_identity
    int x0_identity;   // X_0 = I (V == K)
    float* starts;     // [S][H][K][V] or null: X_0 .. X_{S-1}
    float* end;        // [H][K][V] or null: X_S
};

// Up to two folds over the same transitions in one launch (the composed transition and the
// offset fold of a span are independent): column blocks [0, nx0) run job 0, the rest job 1.
struct FoldParams {
    int S, H, K;
    const float* A;    // [S][H][K][K]
    int nx0;
    FoldJob job0, job1;
};

__device__ __forceinline__ void fold_cp16(void* dst, const void* src) {
    const unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(dst));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(src) : "memory");
}
__device__ __forceinline__ void fold_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void fold_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }

// x = hi + lo with hi, lo tf32 (round to nearest): hi carries the top 11 bits of the significand,
// lo the next 11, so hi*hi' + hi*lo' + lo*hi' reproduces an f32 product to about 2^-22.
__device__ __forceinline__ void split_tf32(float x, uint32_t& hi, uint32_t& lo) {
    hi = to_tf32(x);
    lo = to_tf32(x - __uint_as_float(hi));
}

// X_{s+1} = A_s X_s + B_s for s = 0 .. S-1, one CTA of 8 warps per (COLS columns, head).  The step
// is a dependency chain, so the next transition loads by cp.async (one warp per row, a lane per
// 16 bytes) while step s computes, and the next offsets into registers.  The K x K by K x COLS
// product runs on mma.sync m16n8k8 tf32 with each operand split into two tf32 parts (three products
// per tile, the lo x lo term dropped), accumulating in f32 from the offset: about f32 accuracy (the
// fold's errors reach every later state).  On CUDA cores the same product is bound by shared-memory
// wavefronts (every 16-byte load costs four, broadcast or not); the fragments here cost one per
// 32 values.  Warp w owns rows [16 w, 16 w + 16) and every column of the block.  X is kept in
// shared memory as its two tf32 parts, split once when a step's result is written back (every warp
// reads every row of X, so splitting at the read repeated the work eight times); the starts and
// the end state are stored from the f32 accumulators.
template <int COLS>
__global__ void __launch_bounds__(256, 1) span_fold_kernel(const FoldParams p) {
    constexpr int NT = COLS / 8;      // n-tiles of 8 columns
    constexpr int LDX = COLS + 8;     // X row stride: B fragments (4 rows x 8 columns) conflict-free
    extern __shared__ __align__(16) float fold_smem[];
    float* sA = fold_smem;                                                   // [kFoldStages][128][kFoldLdA]
    uint32_t* sXh = reinterpret_cast<uint32_t*>(sA + kFoldStages * 128 * kFoldLdA);  // [128][LDX] tf32 hi
    uint32_t* sXl = sXh + 128 * LDX;                                         // [128][LDX] tf32 lo
    const bool second = static_cast<int>(blockIdx.x) >= p.nx0;
    const int bx = second ? blockIdx.x - p.nx0 : blockIdx.x;
    const int V = second ? p.job1.V : p.job0.V;
    const float* Bp = second ? p.job1.B : p.job0.B;
    const float* X0 = second ? p.job1.X0 : p.job0.X0;
    const int ident = second ? p.job1.x0_identity : p.job0.x0_identity;
    float* starts = second ? p.job1.starts : p.job0.starts;
    float* endp = second ? p.job1.end : p.job0.end;
    const int h = blockIdx.y, c0 = bx * COLS, K = p.K, S = p.S;
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31, g = lane >> 2, t4 = lane & 3;
    const int r0 = 16 * warp + g;  // accumulator rows r0 and r0 + 8
    const bool act = 16 * warp < K;
    const size_t xb = (size_t)h * K * V;

    auto stage = [&](int s) {
        const float* As = p.A + ((size_t)s * p.H + h) * K * K;
        float* dA = sA + (s % kFoldStages) * (128 * kFoldLdA);
        const int q4 = K >> 2;  // 16-byte pieces per row, <= 32
        if (lane < q4)
            for (int r = warp; r < K; r += 8) fold_cp16(dA + r * kFoldLdA + 4 * lane, As + (size_t)r * K + 4 * lane);
        fold_commit();  // one group per stage on every thread, empty or not
    };
    // the offsets of step s at this thread's accumulator positions (rows r0, r0 + 8; columns
    // 8 nt + 2 t4, + 1)
    auto load_b = [&](int s, float2 (&bb)[NT][2]) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) bb[nt][0] = bb[nt][1] = make_float2(0.f, 0.f);
        if (!Bp || !act) return;
        const float* Bs = Bp + ((size_t)s * p.H + h) * K * V + c0 + 2 * t4;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            bb[nt][0] = *reinterpret_cast<const float2*>(Bs + (size_t)r0 * V + 8 * nt);
            bb[nt][1] = *reinterpret_cast<const float2*>(Bs + (size_t)(r0 + 8) * V + 8 * nt);
        }
    };

    float2 bnext[NT][2];
    if (S > 0) {
        stage(0);
        load_b(0, bnext);
    }
    for (int e = t; e < K * COLS; e += 256) {
        const int r = e / COLS, c = e % COLS;
        float x = 0.f;
        if (ident) x = (r == c0 + c) ? 1.f : 0.f;
        else if (X0) x = X0[xb + (size_t)r * V + c0 + c];
        if (S > 0 && starts) starts[xb + (size_t)r * V + c0 + c] = x;  // X_0, the start of segment 0
        if (S == 0 && endp) endp[xb + (size_t)r * V + c0 + c] = x;
        split_tf32(x, sXh[r * LDX + c], sXl[r * LDX + c]);
    }
    for (int s = 0; s < S; ++s) {
        fold_wait<0>();   // this thread's copies of A_s
        __syncthreads();  // every thread's copies of A_s, and X_s
        if (s + 1 < S) stage(s + 1);  // its slot held A_{s-1}, last read before the barrier above
        float c[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            c[nt][0] = bnext[nt][0].x, c[nt][1] = bnext[nt][0].y;
            c[nt][2] = bnext[nt][1].x, c[nt][3] = bnext[nt][1].y;
        }
        if (s + 1 < S) load_b(s + 1, bnext);
        if (act) {
            const float* Aw = sA + (s % kFoldStages) * (128 * kFoldLdA) + r0 * kFoldLdA + t4;
#pragma unroll 4
            for (int ks = 0; ks < K / 8; ++ks) {
                const float* Ar = Aw + 8 * ks;
                uint32_t ah[4], al[4];
                split_tf32(Ar[0], ah[0], al[0]);
                split_tf32(Ar[8 * kFoldLdA], ah[1], al[1]);
                split_tf32(Ar[4], ah[2], al[2]);
                split_tf32(Ar[8 * kFoldLdA + 4], ah[3], al[3]);
                const int xo = (8 * ks + t4) * LDX + g;
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    const uint32_t bh0 = sXh[xo + 8 * nt], bh1 = sXh[xo + 4 * LDX + 8 * nt];
                    const uint32_t bl0 = sXl[xo + 8 * nt], bl1 = sXl[xo + 4 * LDX + 8 * nt];
                    mma_tf32_16x8x8(c[nt], al[0], al[1], al[2], al[3], bh0, bh1);
                    mma_tf32_16x8x8(c[nt], ah[0], ah[1], ah[2], ah[3], bl0, bl1);
                    mma_tf32_16x8x8(c[nt], ah[0], ah[1], ah[2], ah[3], bh0, bh1);
                }
            }
        }
        __syncthreads();  // every read of X_s is done
        if (act) {
            // X_{s+1}: the start of segment s + 1 (or the end state after the last step) from the
            // f32 accumulators, and its tf32 parts for the next step's products
            float* dst = s + 1 < S ? (starts ? starts + ((size_t)(s + 1) * p.H + h) * K * V : nullptr)
                                   : (endp ? endp + xb : nullptr);
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                const int col = 8 * nt + 2 * t4;
                if (dst) {
                    *reinterpret_cast<float2*>(dst + (size_t)r0 * V + c0 + col) = make_float2(c[nt][0], c[nt][1]);
                    *reinterpret_cast<float2*>(dst + (size_t)(r0 + 8) * V + c0 + col) = make_float2(c[nt][2], c[nt][3]);
                }
                if (s + 1 < S) {
                    split_tf32(c[nt][0], sXh[r0 * LDX + col], sXl[r0 * LDX + col]);
                    split_tf32(c[nt][1], sXh[r0 * LDX + col + 1], sXl[r0 * LDX + col + 1]);
                    split_tf32(c[nt][2], sXh[(r0 + 8) * LDX + col], sXl[(r0 + 8) * LDX + col]);
                    split_tf32(c[nt][3], sXh[(r0 + 8) * LDX + col + 1], sXl[(r0 + 8) * LDX + col + 1]);
                }
            }
        }
    }
}

template <int COLS>
constexpr size_t fold_smem_bytes() {
    return sizeof(float) * (kFoldStages * 128 * kFoldLdA + 2 * 128 * (COLS + 8));
}

int fold_check_job(const FoldJob& j, int K) {
    if (j.V <= 0 || j.V % 16 != 0)
        return fail(DBL_ERR_UNSUPPORTED, "span fold: value width must be a positive multiple of 16");
    if (j.x0_identity && j.V != K) return fail(DBL_ERR_INVALID_ARGUMENT, "span fold: identity start needs V == K");
    for (const void* ptr : {static_cast<const void*>(j.B), static_cast<const void*>(j.X0),
                            static_cast<const void*>(j.starts), static_cast<const void*>(j.end)})
        if (ptr && !aligned(ptr, 16)) return fail(DBL_ERR_INVALID_ARGUMENT, "span fold: arrays must be 16-byte aligned");
    return DBL_OK;
}

template <int COLS>
int fold_launch_cols(const FoldParams& p, int nx, cudaStream_t st) {
    constexpr size_t smem = fold_smem_bytes<COLS>();
    cudaError_t e = cudaFuncSetAttribute(span_fold_kernel<COLS>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return cuda_status(e, "span fold: cudaFuncSetAttribute");
    span_fold_kernel<COLS><<<dim3((unsigned)nx, (unsigned)p.H), 256, smem, st>>>(p);
    return launch_status("span_fold_kernel");
}

// One launch for job 0 and, when job1.V > 0, job 1.  Column blocks of 16 while the grid fits the
// device in one wave, else of 32 (half the CTAs, twice the work each).
int fold_launch(FoldParams p, cudaStream_t st) {
    if (p.K <= 0 || p.K > 128 || p.K % 16 != 0 || p.H <= 0 || p.S < 0)
        return fail(DBL_ERR_UNSUPPORTED, "span fold: key width must be a multiple of 16 up to 128");
    if (p.S > 0 && (!p.A || !aligned(p.A, 16)))
        return fail(DBL_ERR_INVALID_ARGUMENT, "span fold: 16-byte aligned transitions are required");
    if (p.H > 65535) return fail(DBL_ERR_UNSUPPORTED, "span fold: at most 65535 heads");
    int rc = fold_check_job(p.job0, p.K);
    if (rc == DBL_OK && p.job1.V > 0) rc = fold_check_job(p.job1, p.K);
    if (rc != DBL_OK) return rc;
    const int w0 = p.job0.V, w1 = p.job1.V;
    int sms = 148, dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const bool wide = (w0 / 16 + w1 / 16) * p.H > sms && w0 % 32 == 0 && w1 % 32 == 0;
    if (wide) {
        p.nx0 = w0 / 32;
        return fold_launch_cols<32>(p, p.nx0 + w1 / 32, st);
    }
    p.nx0 = w0 / 16;
    return fold_launch_cols<16>(p, p.nx0 + w1 / 16, st);
}

// Segment maps and fold scratch of one span: A [S,H,K,K], B [S,H,K,V] (reused for the rescan's
// final states), starts [S,H,K,V].
struct SegLayout {
    size_t off_a, off_b, off_starts, total;
};

SegLayout seg_layout(int64_t S, int64_t H, int64_t K, int64_t V) {
    auto up = [](size_t x) { return (x + 255) / 256 * 256; };
    SegLayout L{};
    L.off_a = 0;
    L.off_b = up(L.off_a + (size_t)S * H * K * K * 4);
    L.off_starts = up(L.off_b + (size_t)S * H * K * V * 4);
    L.total = up(L.off_starts + (size_t)S * H * K * V * 4);
    return L;
}

int sm_count_current(int* out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(out, cudaDevAttrMultiProcessorCount, dev);
    return cuda_status(e, "SM count");
}

// Segments of a span: the largest power of two S with S x heads <= SMs and whole 64-token chunks
// per segment (1 when the span is short or the heads alone fill the device).
int64_t pick_segments(int64_t T, int64_t H, int sms) {
    int64_t s = 1;
    while ((s * 2) * H <= sms && T % (s * 2 * kChunk) == 0) s *= 2;
    return s;
}

int check_span(const dbl_prefill_args* a, const char* who) {
    if (!a) return fail(DBL_ERR_INVALID_ARGUMENT, "%s: null args", who);
    if (a->batch != 1) return fail(DBL_ERR_UNSUPPORTED, "%s: one sequence (batch 1) per span", who);
    if (a->time <= 0 || a->heads <= 0 || a->key_dim <= 0 || a->value_dim <= 0)
        return fail(DBL_ERR_INVALID_ARGUMENT, "%s: GDN-2 requires nonempty axes", who);
    if (!a->q || !a->k || !a->v || !a->alpha || !a->beta)
        return fail(DBL_ERR_INVALID_ARGUMENT, "%s: q, k, v, alpha and beta are required", who);
    return DBL_OK;
}

// `a` viewed as S equal segments of its one sequence: batch S, time T / S, the same memory.
dbl_prefill_args segment_view(const dbl_prefill_args* a, int64_t S) {
    dbl_prefill_args v = *a;
    const int64_t Ts = a->time / S;
    const int64_t dk[4] = {a->batch, a->time, a->heads, a->key_dim};
    const int64_t dv[4] = {a->batch, a->time, a->heads, a->value_dim};
    const int64_t dg[3] = {a->batch, a->time, a->heads};
    int64_t st[4];
    resolve_strides(a->q_stride, dk, 4, st);
    v.q_stride[0] = Ts * st[1], v.q_stride[1] = st[1], v.q_stride[2] = st[2], v.q_stride[3] = st[3];
    resolve_strides(a->k_stride, dk, 4, st);
    v.k_stride[0] = Ts * st[1], v.k_stride[1] = st[1], v.k_stride[2] = st[2], v.k_stride[3] = st[3];
    resolve_strides(a->v_stride, dv, 4, st);
    v.v_stride[0] = Ts * st[1], v.v_stride[1] = st[1], v.v_stride[2] = st[2], v.v_stride[3] = st[3];
    resolve_strides(a->out_stride, dv, 4, st);
    v.out_stride[0] = Ts * st[1], v.out_stride[1] = st[1], v.out_stride[2] = st[2], v.out_stride[3] = st[3];
    resolve_strides(a->alpha_stride, dg, 3, st);
    v.alpha_stride[0] = Ts * st[1], v.alpha_stride[1] = st[1], v.alpha_stride[2] = st[2];
    resolve_strides(a->beta_stride, dg, 3, st);
    v.beta_stride[0] = Ts * st[1], v.beta_stride[1] = st[1], v.beta_stride[2] = st[2];
    v.batch = S;
    v.time = Ts;
    // valid / reset are [1, T] contiguous, i.e. already [S, T / S] contiguous
    v.initial_state = nullptr;
    v.final_state = nullptr;
    v.out = nullptr;
    return v;
}

// Pass 1: the maps of every segment into the workspace.
int segment_maps(const dbl_prefill_args* a, int64_t S, unsigned char* ws, const SegLayout& L, cudaStream_t st) {
    dbl_prefill_args v = segment_view(a, S);
    float* A = reinterpret_cast<float*>(ws + L.off_a);
    float* Bm = reinterpret_cast<float*>(ws + L.off_b);
    int rc = prefill_dispatch(&v, 1, A, st);
    if (rc != DBL_OK) return rc;
    v.final_state = Bm;
    return prefill_dispatch(&v, 0, nullptr, st);
}

// Fold of the segment maps from `start` (null = zeros) into the segment starts; `end` (optional)
// receives the state after the last segment.
int segment_starts(const dbl_prefill_args* a, int64_t S, unsigned char* ws, const SegLayout& L, const float* start,
                   float* end, cudaStream_t st) {
    FoldParams f{};
    f.S = (int)S, f.H = (int)a->heads, f.K = (int)a->key_dim;
    f.A = reinterpret_cast<const float*>(ws + L.off_a);
    f.job0.V = (int)a->value_dim;
    f.job0.B = reinterpret_cast<const float*>(ws + L.off_b);
    f.job0.X0 = start;
    f.job0.starts = reinterpret_cast<float*>(ws + L.off_starts);
    f.job0.end = end;
    return fold_launch(f, st);
}

// Pass 2: every segment rescanned from its start state; the last segment's final state goes to
// a->final_state.
int segment_rescan(const dbl_prefill_args* a, int64_t S, unsigned char* ws, const SegLayout& L, cudaStream_t st) {
    dbl_prefill_args v = segment_view(a, S);
    v.initial_state = reinterpret_cast<const float*>(ws + L.off_starts);
    v.out = a->out;
    float* fin = reinterpret_cast<float*>(ws + L.off_b);  // the offsets are consumed by the fold
    v.final_state = a->final_state ? fin : nullptr;
    int rc = prefill_dispatch(&v, 0, nullptr, st);
    if (rc != DBL_OK || !a->final_state) return rc;
    const size_t state = (size_t)a->heads * a->key_dim * a->value_dim;
    return cuda_status(cudaMemcpyAsync(a->final_state, fin + (size_t)(S - 1) * state, state * sizeof(float),
                                       cudaMemcpyDeviceToDevice, st),
                       "segmented prefill: final state");
}

// Tokens [t0, t0 + batch x time) of `a`'s one sequence as `batch` consecutive segments of `time`
// tokens: the same memory through offset pointers and strides.  initial_state and final_state
// are cleared (the caller sets them); out keeps its offset when present.
dbl_prefill_args span_view(const dbl_prefill_args* a, int64_t t0, int64_t batch, int64_t time) {
    dbl_prefill_args v = *a;
    const int64_t dk[4] = {a->batch, a->time, a->heads, a->key_dim};
    const int64_t dv[4] = {a->batch, a->time, a->heads, a->value_dim};
    const int64_t dg[3] = {a->batch, a->time, a->heads};
    const size_t es = dtype_size(a->dtype);
    int64_t st[4];
    resolve_strides(a->q_stride, dk, 4, st);
    v.q = static_cast<const unsigned char*>(a->q) + (size_t)(t0 * st[1]) * es;
    v.q_stride[0] = time * st[1], v.q_stride[1] = st[1], v.q_stride[2] = st[2], v.q_stride[3] = st[3];
    resolve_strides(a->k_stride, dk, 4, st);
    v.k = static_cast<const unsigned char*>(a->k) + (size_t)(t0 * st[1]) * es;
    v.k_stride[0] = time * st[1], v.k_stride[1] = st[1], v.k_stride[2] = st[2], v.k_stride[3] = st[3];
    resolve_strides(a->v_stride, dv, 4, st);
    v.v = static_cast<const unsigned char*>(a->v) + (size_t)(t0 * st[1]) * es;
    v.v_stride[0] = time * st[1], v.v_stride[1] = st[1], v.v_stride[2] = st[2], v.v_stride[3] = st[3];
    resolve_strides(a->out_stride, dv, 4, st);
    v.out = a->out ? static_cast<unsigned char*>(a->out) + (size_t)(t0 * st[1]) * es : nullptr;
    v.out_stride[0] = time * st[1], v.out_stride[1] = st[1], v.out_stride[2] = st[2], v.out_stride[3] = st[3];
    resolve_strides(a->alpha_stride, dg, 3, st);
    v.alpha = a->alpha + t0 * st[1];
    v.alpha_stride[0] = time * st[1], v.alpha_stride[1] = st[1], v.alpha_stride[2] = st[2];
    resolve_strides(a->beta_stride, dg, 3, st);
    v.beta = a->beta + t0 * st[1];
    v.beta_stride[0] = time * st[1], v.beta_stride[1] = st[1], v.beta_stride[2] = st[2];
    // valid / reset are [1, T] contiguous, so [batch, time] contiguous from token t0
    v.valid = a->valid ? a->valid + t0 : nullptr;
    v.reset = a->reset ? a->reset + t0 : nullptr;
    v.batch = batch;
    v.time = time;
    v.initial_state = nullptr;
    v.final_state = nullptr;
    return v;
}

// The one-device schedule with a lead segment.  The sequence is cut into a lead segment of t0
// tokens and m segments of lt tokens.  The lead segment needs no span maps: it is scanned from
// the initial state, with its outputs, on a side stream while the maps of segments 1 .. m-1 (two
// launches of (m - 1) x H CTAs) run on the caller's stream; segment m needs no maps either.  The
// fold then gives the starts of segments 1 .. m and one launch of m x H CTAs rescans them.  With
// t0 about 1.8 lt the lead scan ends with the two map launches, so the step takes about three
// scans of lt tokens, against three scans of T / S tokens for S equal segments (m x H <= SMs:
// m = 9 at H = 16 on 148 SMs, lt = T / 10.8 against T / 8).
struct LeadPlan {
    int64_t m = 0, lt = 0, t0 = 0;
};

bool plan_lead(int64_t T, int64_t H, int sms, LeadPlan* out) {
    if (T % kChunk != 0 || H <= 0) return false;
    const int64_t n = T / kChunk;
    for (int64_t m = sms / H; m >= 2; --m) {
        // lt = ceil(n / (m + 1.8)) chunks: the lead scan writes outputs (about 4.5 us per chunk
        // against 4.06 for a map launch on B200), so 1.8 lt of it end with the two map launches
        const int64_t L = (5 * n + 5 * m + 8) / (5 * m + 9);
        const int64_t l0 = n - m * L;  // <= 1.8 L + 1 by the choice of L
        if (L >= 1 && l0 >= 1) {
            out->m = m;
            out->lt = L * kChunk;
            out->t0 = l0 * kChunk;
            return true;
        }
    }
    return false;
}

// One side stream and its fork / join events per device, created on first use and kept for the
// life of the process.  The fork, the side launches and the join are issued under g_side_mu, so
// concurrent callers on one device cannot interleave their event records.
struct SideStream {
    cudaStream_t s = nullptr;
    cudaEvent_t fork = nullptr, join = nullptr;
};
std::mutex g_side_mu;
SideStream g_side[64];

int side_stream(SideStream** out) {
    int dev = 0;
    int rc = cuda_status(cudaGetDevice(&dev), "side stream: cudaGetDevice");
    if (rc != DBL_OK) return rc;
    if (dev < 0 || dev >= 64) return fail(DBL_ERR_UNSUPPORTED, "side stream: device index %d out of range", dev);
    SideStream& ss = g_side[dev];
    if (!ss.s) {
        rc = cuda_status(cudaStreamCreateWithFlags(&ss.s, cudaStreamNonBlocking), "side stream: create");
        if (rc == DBL_OK) rc = cuda_status(cudaEventCreateWithFlags(&ss.fork, cudaEventDisableTiming), "side stream: event");
        if (rc == DBL_OK) rc = cuda_status(cudaEventCreateWithFlags(&ss.join, cudaEventDisableTiming), "side stream: event");
        if (rc != DBL_OK) return rc;
    }
    *out = &ss;
    return DBL_OK;
}

int lead_prefill(const dbl_prefill_args* a, const LeadPlan& P, unsigned char* ws, const SegLayout& L, cudaStream_t st) {
    const size_t state = (size_t)a->heads * a->key_dim * a->value_dim;
    float* A = reinterpret_cast<float*>(ws + L.off_a);
    float* Bm = reinterpret_cast<float*>(ws + L.off_b);
    float* starts = reinterpret_cast<float*>(ws + L.off_starts);
    int rc = DBL_OK;
    {
        std::lock_guard<std::mutex> lock(g_side_mu);
        SideStream* ss = nullptr;
        rc = side_stream(&ss);
        if (rc != DBL_OK) return rc;
        rc = cuda_status(cudaEventRecord(ss->fork, st), "lead prefill: fork");
        if (rc == DBL_OK) rc = cuda_status(cudaStreamWaitEvent(ss->s, ss->fork, 0), "lead prefill: fork");
        if (rc != DBL_OK) return rc;
        // the lead segment: initial state -> outputs of tokens [0, t0) and the start of segment 1
        dbl_prefill_args v0 = span_view(a, 0, 1, P.t0);
        v0.initial_state = a->initial_state;
        v0.final_state = starts;
        const int rc_side = prefill_dispatch(&v0, 0, nullptr, ss->s);
        // the maps of segments 1 .. m-1
        dbl_prefill_args vm = span_view(a, P.t0, P.m - 1, P.lt);
        vm.out = nullptr;
        rc = prefill_dispatch(&vm, 1, A, st);
        if (rc == DBL_OK) {
            vm.final_state = Bm;
            rc = prefill_dispatch(&vm, 0, nullptr, st);
        }
        // join even after a failed launch, so that nothing queued on the side stream outlives the call
        const int rc_join = cuda_status(cudaEventRecord(ss->join, ss->s), "lead prefill: join");
        const int rc_wait = rc_join == DBL_OK ? cuda_status(cudaStreamWaitEvent(st, ss->join, 0), "lead prefill: join") : rc_join;
        if (rc == DBL_OK) rc = rc_side;
        if (rc == DBL_OK) rc = rc_wait;
        if (rc != DBL_OK) return rc;
    }
    // X_0 = the start of segment 1; X_{s+1} = A_s X_s + B_s over the maps of segments 1 .. m-1
    FoldParams f{};
    f.S = (int)(P.m - 1), f.H = (int)a->heads, f.K = (int)a->key_dim;
    f.A = A;
    f.job0.V = (int)a->value_dim;
    f.job0.B = Bm;
    f.job0.X0 = starts;
    f.job0.starts = starts;
    f.job0.end = starts + (size_t)(P.m - 1) * state;
    rc = fold_launch(f, st);
    if (rc != DBL_OK) return rc;
    // segments 1 .. m from their starts
    dbl_prefill_args vr = span_view(a, P.t0, P.m, P.lt);
    vr.initial_state = starts;
    vr.final_state = a->final_state ? Bm : nullptr;  // the offsets are consumed by the fold
    rc = prefill_dispatch(&vr, 0, nullptr, st);
    if (rc != DBL_OK || !a->final_state) return rc;
    return cuda_status(cudaMemcpyAsync(a->final_state, Bm + (size_t)(P.m - 1) * state, state * sizeof(float),
                                       cudaMemcpyDeviceToDevice, st),
                       "segmented prefill: final state");
}

// segments = 0: the lead schedule when it applies (plan_lead), else 0 is resolved by
// pick_segments as for explicit equal segments.
int lead_plan_for(const dbl_prefill_args* a, int64_t segments, LeadPlan* P) {
    if (segments != 0) return 0;
    int sms = 0;
    if (sm_count_current(&sms) != DBL_OK) return 0;
    return plan_lead(a->time, a->heads, sms, P) ? 1 : 0;
}

int resolve_segments(const dbl_prefill_args* a, int64_t segments, int64_t* out) {
    int64_t S = segments;
    if (S == 0) {
        int sms = 0;
        int rc = sm_count_current(&sms);
        if (rc != DBL_OK) return rc;
        S = pick_segments(a->time, a->heads, sms);
    }
    if (S < 1 || a->time % S != 0)
        return fail(DBL_ERR_INVALID_ARGUMENT, "segmented prefill: %lld segments do not divide %lld tokens",
                    (long long)S, (long long)a->time);
    *out = S;
    return DBL_OK;
}

}  // namespace
}  // namespace dbl

extern "C" int dbl_gdn2_span_fold(const float* transition, const float* offset, int64_t segments, int64_t heads,
                                  int64_t key_dim, int64_t value_dim, const float* start, float* starts, float* end,
                                  float* composed_transition, dbl_stream_t stream) {
    using namespace dbl;
    if (segments < 0 || heads <= 0 || key_dim <= 0 || value_dim <= 0)
        return fail(DBL_ERR_INVALID_ARGUMENT, "span fold: nonempty heads and widths, segments >= 0");
    if (segments > 0x7fffffff || heads > 0x7fffffff)
        return fail(DBL_ERR_UNSUPPORTED, "span fold: axis exceeds 32-bit limits");
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    FoldParams f{};
    f.S = (int)segments, f.H = (int)heads, f.K = (int)key_dim;
    f.A = transition;
    // the composed transition (identity start, no offsets) and the offset fold share one launch
    FoldJob comp{}, fold{};
    if (composed_transition) {
        comp.V = (int)key_dim;
        comp.x0_identity = 1;
        comp.end = composed_transition;
    }
    if (starts || end) {
        fold.V = (int)value_dim;
        fold.B = offset;
        fold.X0 = start;
        fold.starts = starts;
        fold.end = end;
    }
    if (comp.V > 0) {
        f.job0 = comp;
        f.job1 = fold;
    } else if (fold.V > 0) {
        f.job0 = fold;
    } else {
        return DBL_OK;
    }
    return fold_launch(f, st);
}

extern "C" size_t dbl_gdn2_prefill_segmented_workspace_bytes(const dbl_prefill_args* a, int64_t segments) {
    using namespace dbl;
    if (check_span(a, "segmented prefill") != DBL_OK) return 0;
    LeadPlan P;
    if (lead_plan_for(a, segments, &P)) return seg_layout(P.m, a->heads, a->key_dim, a->value_dim).total;
    int64_t S = 0;
    if (resolve_segments(a, segments, &S) != DBL_OK) return 0;
    return seg_layout(S, a->heads, a->key_dim, a->value_dim).total;
}

extern "C" int dbl_gdn2_prefill_segmented(const dbl_prefill_args* a, int64_t segments, void* workspace,
                                          size_t workspace_bytes, dbl_stream_t stream) {
    using namespace dbl;
    int rc = check_span(a, "segmented prefill");
    if (rc != DBL_OK) return rc;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    LeadPlan P;
    if (lead_plan_for(a, segments, &P)) {
        const SegLayout L = seg_layout(P.m, a->heads, a->key_dim, a->value_dim);
        if (!workspace || workspace_bytes < L.total)
            return fail(DBL_ERR_WORKSPACE, "segmented prefill: workspace of %zu bytes required (got %zu)", L.total,
                        workspace_bytes);
        if (!aligned(workspace, 256)) return fail(DBL_ERR_INVALID_ARGUMENT, "segmented prefill: workspace must be 256-byte aligned");
        return lead_prefill(a, P, static_cast<unsigned char*>(workspace), L, st);
    }
    int64_t S = 0;
    rc = resolve_segments(a, segments, &S);
    if (rc != DBL_OK) return rc;
    if (S == 1) return dbl_gdn2_prefill(a, stream);
    const SegLayout L = seg_layout(S, a->heads, a->key_dim, a->value_dim);
    if (!workspace || workspace_bytes < L.total)
        return fail(DBL_ERR_WORKSPACE, "segmented prefill: workspace of %zu bytes required (got %zu)", L.total,
                    workspace_bytes);
    if (!aligned(workspace, 256)) return fail(DBL_ERR_INVALID_ARGUMENT, "segmented prefill: workspace must be 256-byte aligned");
    unsigned char* ws = static_cast<unsigned char*>(workspace);
    rc = segment_maps(a, S, ws, L, st);
    if (rc == DBL_OK) rc = segment_starts(a, S, ws, L, a->initial_state, nullptr, st);
    if (rc == DBL_OK) rc = segment_rescan(a, S, ws, L, st);
    return rc;
}

// ------------------------------------------------------------------------------ multi-device
namespace dbl {
namespace {

// Per-device workspace: the segment layout, then the span map slots of every device
// (transition [n][H][K][K], offset [n][H][K][V]; slot 0's offset is device 0's end state) and the
// device's start state [H][K][V].
struct ShardLayout {
    SegLayout seg;
    size_t off_ga, off_gb, off_sin, total;
};

ShardLayout shard_layout(int64_t S, int n, int64_t H, int64_t K, int64_t V) {
    auto up = [](size_t x) { return (x + 255) / 256 * 256; };
    ShardLayout L{};
    L.seg = seg_layout(S, H, K, V);
    L.off_ga = L.seg.total;
    L.off_gb = up(L.off_ga + (size_t)n * H * K * K * 4);
    L.off_sin = up(L.off_gb + (size_t)n * H * K * V * 4);
    L.total = up(L.off_sin + (size_t)H * K * V * 4);
    return L;
}

// Restores the calling thread's device when the multi-device call returns.
struct DeviceGuard {
    int saved = -1;
    DeviceGuard() { cudaGetDevice(&saved); }
    ~DeviceGuard() {
        if (saved >= 0) cudaSetDevice(saved);
    }
};

}  // namespace
}  // namespace dbl

extern "C" size_t dbl_gdn2_prefill_time_sharded_workspace_bytes(const dbl_prefill_args* span, int n_gpus,
                                                                 int64_t segments) {
    using namespace dbl;
    if (n_gpus < 1 || check_span(span, "time-sharded prefill") != DBL_OK) return 0;
    int64_t S = 0;
    if (resolve_segments(span, segments, &S) != DBL_OK) return 0;
    return shard_layout(S, n_gpus, span->heads, span->key_dim, span->value_dim).total;
}

extern "C" int dbl_gdn2_prefill_time_sharded(const dbl_prefill_args* spans, int n_gpus, const int* devices,
                                             dbl_stream_t const* streams, int64_t segments, void* const* workspaces,
                                             const size_t* workspace_bytes) {
    using namespace dbl;
    if (!spans || !devices || !streams || !workspaces || !workspace_bytes || n_gpus < 1)
        return fail(DBL_ERR_INVALID_ARGUMENT, "time-sharded prefill: spans, devices, streams and workspaces are required");
    const int64_t H = spans[0].heads, K = spans[0].key_dim, V = spans[0].value_dim;
    for (int g = 0; g < n_gpus; ++g) {
        int rc = check_span(&spans[g], "time-sharded prefill");
        if (rc != DBL_OK) return rc;
        if (spans[g].heads != H || spans[g].key_dim != K || spans[g].value_dim != V || spans[g].dtype != spans[0].dtype)
            return fail(DBL_ERR_INVALID_ARGUMENT, "time-sharded prefill: every span needs the same heads, widths and dtype");
    }
    std::vector<int64_t> S(n_gpus);
    std::vector<ShardLayout> L(n_gpus);
    DeviceGuard guard;
    for (int g = 0; g < n_gpus; ++g) {
        int rc = cuda_status(cudaSetDevice(devices[g]), "time-sharded prefill: cudaSetDevice");
        if (rc == DBL_OK) rc = resolve_segments(&spans[g], segments, &S[g]);
        if (rc != DBL_OK) return rc;
        L[g] = shard_layout(S[g], n_gpus, H, K, V);
        if (!workspaces[g] || workspace_bytes[g] < L[g].total)
            return fail(DBL_ERR_WORKSPACE, "time-sharded prefill: device %d needs a workspace of %zu bytes (got %zu)", g,
                        L[g].total, workspace_bytes[g]);
        if (!aligned(workspaces[g], 256))
            return fail(DBL_ERR_INVALID_ARGUMENT, "time-sharded prefill: workspaces must be 256-byte aligned");
    }
    const size_t tbytes = (size_t)H * K * K * 4, obytes = (size_t)H * K * V * 4;
    std::vector<cudaEvent_t> ready(n_gpus, nullptr);
    auto cleanup = [&](int rc) {
        for (cudaEvent_t e : ready)
            if (e) cudaEventDestroy(e);
        return rc;
    };
    // pass 1 and the span maps (device 0: its end state) on every device
    for (int g = 0; g < n_gpus; ++g) {
        unsigned char* ws = static_cast<unsigned char*>(workspaces[g]);
        cudaStream_t st = reinterpret_cast<cudaStream_t>(streams[g]);
        int rc = cuda_status(cudaSetDevice(devices[g]), "time-sharded prefill: cudaSetDevice");
        if (rc == DBL_OK) rc = segment_maps(&spans[g], S[g], ws, L[g].seg, st);
        float* ga = reinterpret_cast<float*>(ws + L[g].off_ga) + (size_t)g * H * K * K;
        float* gb = reinterpret_cast<float*>(ws + L[g].off_gb) + (size_t)g * H * K * V;
        if (rc == DBL_OK && g == 0) {
            rc = segment_starts(&spans[0], S[0], ws, L[0].seg, spans[0].initial_state, gb, st);
        } else if (rc == DBL_OK) {
            rc = dbl_gdn2_span_fold(reinterpret_cast<const float*>(ws + L[g].seg.off_a),
                                    reinterpret_cast<const float*>(ws + L[g].seg.off_b), S[g], H, K, V, nullptr, nullptr,
                                    gb, ga, streams[g]);
        }
        if (rc == DBL_OK) rc = cuda_status(cudaEventCreateWithFlags(&ready[g], cudaEventDisableTiming), "event");
        if (rc == DBL_OK) rc = cuda_status(cudaEventRecord(ready[g], st), "event record");
        if (rc != DBL_OK) return cleanup(rc);
    }
    // hand-off: device g pulls the map slots of devices 0 .. g-1, folds its start state, then runs
    // its own fold and the rescan
    for (int g = 0; g < n_gpus; ++g) {
        unsigned char* ws = static_cast<unsigned char*>(workspaces[g]);
        cudaStream_t st = reinterpret_cast<cudaStream_t>(streams[g]);
        int rc = cuda_status(cudaSetDevice(devices[g]), "time-sharded prefill: cudaSetDevice");
        float* ga = reinterpret_cast<float*>(ws + L[g].off_ga);
        float* gb = reinterpret_cast<float*>(ws + L[g].off_gb);
        for (int r = 0; r < g && rc == DBL_OK; ++r) {
            const unsigned char* src = static_cast<const unsigned char*>(workspaces[r]);
            rc = cuda_status(cudaStreamWaitEvent(st, ready[r], 0), "time-sharded prefill: wait for device");
            if (rc == DBL_OK && r > 0)
                rc = cuda_status(cudaMemcpyPeerAsync(ga + (size_t)r * H * K * K, devices[g],
                                                     src + L[r].off_ga + (size_t)r * tbytes, devices[r], tbytes, st),
                                 "time-sharded prefill: transition hand-off");
            if (rc == DBL_OK)
                rc = cuda_status(cudaMemcpyPeerAsync(gb + (size_t)r * H * K * V, devices[g],
                                                     src + L[r].off_gb + (size_t)r * obytes, devices[r], obytes, st),
                                 "time-sharded prefill: state hand-off");
        }
        if (rc != DBL_OK) return cleanup(rc);
        if (g > 0) {
            // S_in(g) = fold of the maps of devices 1 .. g-1 from device 0's end state
            float* sin = reinterpret_cast<float*>(ws + L[g].off_sin);
            rc = dbl_gdn2_span_fold(ga + (size_t)H * K * K, gb + (size_t)H * K * V, g - 1, H, K, V, gb, nullptr, sin,
                                    nullptr, streams[g]);
            if (rc == DBL_OK) rc = segment_starts(&spans[g], S[g], ws, L[g].seg, sin, nullptr, st);
            if (rc != DBL_OK) return cleanup(rc);
        }
        rc = segment_rescan(&spans[g], S[g], ws, L[g].seg, st);
        if (rc != DBL_OK) return cleanup(rc);
    }
    return cleanup(DBL_OK);
}
