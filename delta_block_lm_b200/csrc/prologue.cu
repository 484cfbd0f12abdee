// GDN-2 mixer prologue: the work between the projections and the scan, fused into one pass.
//
// Replaces, for MixerKind::Gdn2, the gate and input producer of Mixer::forward_inner
// (crates/mixers/src/lib.rs:446-528) with its kernels:
//   q, k = l2(silu(conv(proj)))    conv: depthwise causal, one document (conv.rs:7-45);
//                                  l2: x / sqrt(sum x^2 + 1e-6) per head row (norm.rs:23-80, mode 0)
//   v    = silu(conv(proj_v))
//   alpha = exp(-softplus(proj_decay + bias[h,k]) exp(scale[h]))   softplus threshold 20 (decay.rs:13-34)
//   erase, write = sigmoid(proj)
// Documents are cumsum(reset * valid) over time (lib.rs:451-455); a conv lag contributes only when
// its source token is in the destination's document, i.e. no valid reset lies in (source, dest],
// and both tokens are valid -- decided locally, without the cumulative sum.
//
// One CTA per (b, h, tile of TT tokens), HBM-bound, so the layout is chosen for bytes in flight:
//   1. cp.async (16 B each, no register round trip) stages the tile's q, k and v projection rows
//      plus the W - 1 earlier tokens of the conv halo, raw in the input dtype, and the head's conv
//      weights into shared memory;
//   2. while those land, the gates stream: each thread loads 8-element units of every gate input
//      it owns before it stores any output (loads and stores may alias as far as the compiler
//      knows, so the order is written out);
//   3. a warp per token convolves from shared memory with each lane on 4 consecutive channels,
//      applies silu and the L2 row norm (warp shuffles) and stores 4 channels at a time.
// Widths that are not multiples of 8 or pointers that are not 16-byte aligned take the same
// kernel with element-wise staging and single channels per lane.
//
// At these sizes the kernel issues more instructions than it moves bytes, so the transcendental
// parts use the hardware approximations: sigmoid(x) = 1 / (1 + e^-x) and silu(x) = x / (1 + e^-x)
// with __expf and __fdividef (a few ulp), and the decay gate with softplus(z) =
// max(z, 0) + log1p(e^-|z|), log1p from the atanh series (see log1p_unit).  The f64 oracle bounds
// the result to 1e-6 absolute on the gates (values in [0, 1]).
#include "common.cuh"

namespace dbl {
namespace {

constexpr int MAXW = 8;     // conv width limit
constexpr int MAXC = 256;   // key / value width limit
constexpr int TT = 32;      // tokens per CTA
constexpr int THREADS = 256;

struct ProParams {
    int B, T, H, K, V, W;
    const void *pq, *pk, *pv, *pd, *pe, *pw;
    const float *cq, *ck, *cv, *bias, *scale, *valid, *reset;
    void *q, *k, *v;
    float *alpha, *erase, *write;
};

// shared-memory carve-up, identical on host and device; every region starts on 16 bytes
struct Layout {
    size_t xq, xk, xv, wq, wk, wv, sv, sr, mask, total;
};
__host__ __device__ __forceinline__ size_t rnd16(size_t x) { return (x + 15) & ~size_t(15); }
__host__ __device__ __forceinline__ Layout layout(int K, int V, int W, int es) {
    const size_t rows = TT + W - 1;
    Layout L{};
    size_t o = 0;
    L.xq = o; o += rnd16(rows * K * es);
    L.xk = o; o += rnd16(rows * K * es);
    L.xv = o; o += rnd16(rows * V * es);
    L.wq = o; o += rnd16((size_t)W * K * 4);
    L.wk = o; o += rnd16((size_t)W * K * 4);
    L.wv = o; o += rnd16((size_t)W * V * 4);
    L.sv = o; o += rnd16(rows * 4);
    L.sr = o; o += rnd16(rows * 4);
    L.mask = o; o += rnd16(TT * 4);
    L.total = o;
    return L;
}

// e^-x overflows to +inf below x = -88.7; __fdividef(., inf) is 0, the correct limit of both
__device__ __forceinline__ float siluf(float x) { return __fdividef(x, 1.f + __expf(-x)); }
// silu(x) = x/2 (1 + tanh(x/2)) on the hardware tanh (one MUFU operation; relative error about
// 2^-11), used only where the result is rounded to bf16 (relative step 2^-8)
__device__ __forceinline__ float silu_bf16out(float x) {
    float th;
    asm("tanh.approx.f32 %0, %1;" : "=f"(th) : "f"(0.5f * x));
    const float hx = 0.5f * x;
    return fmaf(hx, th, hx);
}
__device__ __forceinline__ float sigmoidf(float x) { return __fdividef(1.f, 1.f + __expf(-x)); }

// log1p(v) for v in [0, 1] by log1p(v) = log((1 + s) / (1 - s)) = 2 atanh(s), s = v / (2 + v) in
// [0, 1/3], with the Taylor series atanh(s) = s + s^3/3 + s^5/5 + ...; the first omitted term
// (s^15/15) is below 2^-26 of the sum, so the error is that of the division (2 ulp)
__device__ __forceinline__ float log1p_unit(float v) {
    const float s = __fdividef(v, 2.f + v), s2 = s * s;
    float p = 1.f / 13.f;
    p = fmaf(p, s2, 1.f / 11.f);
    p = fmaf(p, s2, 1.f / 9.f);
    p = fmaf(p, s2, 1.f / 7.f);
    p = fmaf(p, s2, 1.f / 5.f);
    p = fmaf(p, s2, 1.f / 3.f);
    p = fmaf(p, s2, 1.f);
    return 2.f * s * p;
}
// exp(-softplus(z) e^scale) with Burn's threshold: softplus(z) = z above 20, else
// log(1 + e^z) = max(z, 0) + log1p(e^-|z|)
__device__ __forceinline__ float decay_gate(float z, float es) {
    const float sp = z > 20.f ? z : fmaxf(z, 0.f) + log1p_unit(__expf(-fabsf(z)));
    return __expf(-sp * es);
}

__device__ __forceinline__ float warp_sum32(float x) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
    return x;
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    const unsigned s = (unsigned)__cvta_generic_to_shared(dst);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;\n" ::: "memory"); }

template <typename TI>
__device__ __forceinline__ TI zero_in() {
    if constexpr (sizeof(TI) == 4) return 0.f;
    else return __float2bfloat16_rn(0.f);
}

// bf16 -> f32 of the two halves of a 32-bit word (exact: bf16 is the top half of an f32)
__device__ __forceinline__ float bf_lo(unsigned w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf_hi(unsigned w) { return __uint_as_float(w & 0xffff0000u); }

// eight consecutive gate inputs, loaded raw (streaming, read once) and unpacked after the loads
template <typename TI>
struct Pack8;
template <>
struct Pack8<__nv_bfloat16> {
    uint4 u;
    __device__ __forceinline__ void load(const __nv_bfloat16* p) { u = __ldcs(reinterpret_cast<const uint4*>(p)); }
    __device__ __forceinline__ void unpack(float (&x)[8]) const {
        x[0] = bf_lo(u.x); x[1] = bf_hi(u.x); x[2] = bf_lo(u.y); x[3] = bf_hi(u.y);
        x[4] = bf_lo(u.z); x[5] = bf_hi(u.z); x[6] = bf_lo(u.w); x[7] = bf_hi(u.w);
    }
};
template <>
struct Pack8<float> {
    float4 a, b;
    __device__ __forceinline__ void load(const float* p) {
        a = __ldcs(reinterpret_cast<const float4*>(p));
        b = __ldcs(reinterpret_cast<const float4*>(p) + 1);
    }
    __device__ __forceinline__ void unpack(float (&x)[8]) const {
        x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w; x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
    }
};
__device__ __forceinline__ void st8(float* p, const float (&x)[8]) {
    reinterpret_cast<float4*>(p)[0] = make_float4(x[0], x[1], x[2], x[3]);
    reinterpret_cast<float4*>(p)[1] = make_float4(x[4], x[5], x[6], x[7]);
}

// E consecutive elements from shared memory / to global memory
template <typename TI, int E>
__device__ __forceinline__ void lds(const TI* p, float (&x)[E]) {
    static_assert(E == 1 || E == 4, "1 or 4 channels per lane");
    if constexpr (E == 1) x[0] = to_f32(*p);
    else if constexpr (sizeof(TI) == 2) {
        const uint2 w = *reinterpret_cast<const uint2*>(p);
        x[0] = bf_lo(w.x); x[1] = bf_hi(w.x); x[2] = bf_lo(w.y); x[3] = bf_hi(w.y);
    } else {
        const float4 f = *reinterpret_cast<const float4*>(p);
        x[0] = f.x; x[1] = f.y; x[2] = f.z; x[3] = f.w;
    }
}
template <int E>
__device__ __forceinline__ void ldw(const float* p, float (&x)[E]) {
    if constexpr (E == 1) x[0] = *p;
    else {
        const float4 f = *reinterpret_cast<const float4*>(p);
        x[0] = f.x; x[1] = f.y; x[2] = f.z; x[3] = f.w;
    }
}
__device__ __forceinline__ unsigned pack_bf2(float a, float b) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const unsigned*>(&h);
}
template <typename TO, int E>
__device__ __forceinline__ void stg(TO* p, const float (&y)[E], float s) {
    if constexpr (E == 1) {
        if constexpr (sizeof(TO) == 4) *p = y[0] * s;
        else *p = __float2bfloat16_rn(y[0] * s);
    } else if constexpr (sizeof(TO) == 2) {
        *reinterpret_cast<uint2*>(p) = make_uint2(pack_bf2(y[0] * s, y[1] * s), pack_bf2(y[2] * s, y[3] * s));
    } else {
        *reinterpret_cast<float4*>(p) = make_float4(y[0] * s, y[1] * s, y[2] * s, y[3] * s);
    }
}

// rows t0 - W + 1 .. t0 + TT - 1 of one head's C channels of a [B, T, H*C] array into dst [rows][C]
// (zeros outside [0, T))
template <typename TI, bool VEC>
__device__ __forceinline__ void stage_rows(TI* dst, const TI* src, int C, int HC, int h, int b, int T, int t0,
                                           int W, int tid) {
    const int rows = TT + W - 1, tb = t0 - (W - 1);
    if constexpr (VEC) {
        const int cpr = C * (int)sizeof(TI) / 16;  // 16-byte pieces per row
        for (int i = tid; i < rows * cpr; i += THREADS) {
            const int r = i / cpr, j = i - r * cpr, t = tb + r;
            char* d = reinterpret_cast<char*>(dst + (size_t)r * C) + 16 * j;
            if (t >= 0 && t < T)
                cp_async16(d, reinterpret_cast<const char*>(src + ((size_t)b * T + t) * HC + (size_t)h * C) + 16 * j);
            else
                *reinterpret_cast<uint4*>(d) = make_uint4(0u, 0u, 0u, 0u);
        }
    } else {
        for (int i = tid; i < rows * C; i += THREADS) {
            const int r = i / C, c = i - r * C, t = tb + r;
            dst[i] = (t >= 0 && t < T) ? src[((size_t)b * T + t) * HC + (size_t)h * C + c] : zero_in<TI>();
        }
    }
}

// the head's conv weights [W][C] out of [W, H*C]
template <bool VEC>
__device__ __forceinline__ void stage_w(float* dst, const float* src, int C, int HC, int h, int W, int tid) {
    if constexpr (VEC) {
        const int cpr = C / 4;
        for (int i = tid; i < W * cpr; i += THREADS) {
            const int lag = i / cpr, j = i - lag * cpr;
            cp_async16(dst + (size_t)lag * C + 4 * j, src + (size_t)lag * HC + (size_t)h * C + 4 * j);
        }
    } else {
        for (int i = tid; i < W * C; i += THREADS) {
            const int lag = i / C, c = i - lag * C;
            dst[i] = src[(size_t)lag * HC + (size_t)h * C + c];
        }
    }
}

// conv + silu (+ L2 norm) of one token's row: staged row rr, lanes on E-channel groups; bit lag
// of mk says whether that lag contributes (all bits set: the unmasked loop).  WT > 0 fixes the
// conv width at compile time, WT == 0 reads it from W.
template <typename TI, typename TO, int E, int WT, bool NORM>
__device__ __forceinline__ void conv_row(const TI* xs, const float* ws, int C, int Wrt, int rr, unsigned mk,
                                         int lane, TO* out) {
    constexpr int MAXU = MAXC / (32 * E);
    constexpr int WL = WT > 0 ? WT : MAXW;
    const int W = WT > 0 ? WT : Wrt;
    const bool full = mk == (1u << W) - 1u;
    float y[MAXU][E];
    float ss = 0.f;
#pragma unroll
    for (int u = 0; u < MAXU; ++u) {
        const int c = E * (lane + 32 * u);
#pragma unroll
        for (int e = 0; e < E; ++e) y[u][e] = 0.f;
        if (c < C) {
            if (full) {
#pragma unroll
                for (int lag = 0; lag < WL; ++lag) {
                    if (lag < W) {
                        float xv[E], wv[E];
                        lds<TI, E>(xs + (size_t)(rr - lag) * C + c, xv);
                        ldw<E>(ws + lag * C + c, wv);
#pragma unroll
                        for (int e = 0; e < E; ++e) y[u][e] = fmaf(xv[e], wv[e], y[u][e]);
                    }
                }
            } else {
#pragma unroll
                for (int lag = 0; lag < WL; ++lag) {
                    if (lag < W && (mk >> lag & 1u)) {
                        float xv[E], wv[E];
                        lds<TI, E>(xs + (size_t)(rr - lag) * C + c, xv);
                        ldw<E>(ws + lag * C + c, wv);
#pragma unroll
                        for (int e = 0; e < E; ++e) y[u][e] = fmaf(xv[e], wv[e], y[u][e]);
                    }
                }
            }
#pragma unroll
            for (int e = 0; e < E; ++e) {
                if constexpr (sizeof(TO) == 2) y[u][e] = silu_bf16out(y[u][e]);
                else y[u][e] = siluf(y[u][e]);
                ss = fmaf(y[u][e], y[u][e], ss);
            }
        }
    }
    float s = 1.f;
    if constexpr (NORM) s = rsqrtf(warp_sum32(ss) + 1e-6f);
#pragma unroll
    for (int u = 0; u < MAXU; ++u) {
        const int c = E * (lane + 32 * u);
        if (c < C) stg<TO, E>(out + c, y[u], s);
    }
}

// WT > 0 fixes the conv width and CT > 0 the key and value widths (K = V = CT) at compile time, so
// that the index arithmetic of the common shape folds to shifts; 0 reads them from p.
template <typename TI, typename TO, bool VEC, int WT, int CT>
__global__ void __launch_bounds__(THREADS, sizeof(TI) == 2 ? 5 : 3) prologue_kernel(const ProParams p) {
    extern __shared__ __align__(16) unsigned char smraw[];
    constexpr int E = VEC ? 4 : 1;
    const int K = CT > 0 ? CT : p.K, V = CT > 0 ? CT : p.V, W = WT > 0 ? WT : p.W, T = p.T;
    const Layout L = layout(K, V, W, (int)sizeof(TI));
    TI* xq = reinterpret_cast<TI*>(smraw + L.xq);
    TI* xk = reinterpret_cast<TI*>(smraw + L.xk);
    TI* xv = reinterpret_cast<TI*>(smraw + L.xv);
    float* wq = reinterpret_cast<float*>(smraw + L.wq);
    float* wk = reinterpret_cast<float*>(smraw + L.wk);
    float* wv = reinterpret_cast<float*>(smraw + L.wv);
    float* sv = reinterpret_cast<float*>(smraw + L.sv);
    float* sr = reinterpret_cast<float*>(smraw + L.sr);
    const int tiles = (T + TT - 1) / TT;
    const int tile = blockIdx.x % tiles, bh = blockIdx.x / tiles;
    const int h = bh % p.H, b = bh / p.H;
    const int t0 = tile * TT, nt = min(TT, T - t0), tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int HK = p.H * K, HV = p.H * V;

    // 1. asynchronous staging of the conv inputs and weights
    stage_rows<TI, VEC>(xq, static_cast<const TI*>(p.pq), K, HK, h, b, T, t0, W, tid);
    stage_rows<TI, VEC>(xk, static_cast<const TI*>(p.pk), K, HK, h, b, T, t0, W, tid);
    stage_rows<TI, VEC>(xv, static_cast<const TI*>(p.pv), V, HV, h, b, T, t0, W, tid);
    stage_w<VEC>(wq, p.cq, K, HK, h, W, tid);
    stage_w<VEC>(wk, p.ck, K, HK, h, W, tid);
    stage_w<VEC>(wv, p.cv, V, HV, h, W, tid);
    for (int r = tid; r < TT + W - 1; r += THREADS) {
        const int t = t0 - (W - 1) + r;
        const bool in = t >= 0 && t < T;
        sv[r] = in ? p.valid[(size_t)b * T + t] : 0.f;
        sr[r] = in ? p.reset[(size_t)b * T + t] : 0.f;
    }

    // 2. gates, elementwise over the tile's tokens
    const float es = expf(p.scale[h]);
    const TI* pd = static_cast<const TI*>(p.pd);
    const TI* pe = static_cast<const TI*>(p.pe);
    const TI* pw = static_cast<const TI*>(p.pw);
    constexpr int GU = 2;  // gate units (8 elements each) in flight per thread
    if constexpr (VEC) {
        {
            const int upr = K / 8, n = nt * upr;
            for (int u0 = tid; u0 < n; u0 += GU * THREADS) {
                Pack8<TI> d[GU], e[GU];
                size_t g[GU];
#pragma unroll
                for (int s = 0; s < GU; ++s) {
                    const int u = u0 + s * THREADS;
                    if (u < n) {
                        const int r = u / upr, j = u - r * upr;
                        g[s] = ((size_t)b * T + t0 + r) * HK + (size_t)h * K + 8 * j;
                        d[s].load(pd + g[s]);
                        e[s].load(pe + g[s]);
                    }
                }
#pragma unroll
                for (int s = 0; s < GU; ++s) {
                    const int u = u0 + s * THREADS;
                    if (u < n) {
                        const int j = u % upr;
                        float x[8], bb[8], y[8];
                        const float4 b0 = __ldg(reinterpret_cast<const float4*>(p.bias + (size_t)h * K + 8 * j));
                        const float4 b1 = __ldg(reinterpret_cast<const float4*>(p.bias + (size_t)h * K + 8 * j) + 1);
                        bb[0] = b0.x; bb[1] = b0.y; bb[2] = b0.z; bb[3] = b0.w;
                        bb[4] = b1.x; bb[5] = b1.y; bb[6] = b1.z; bb[7] = b1.w;
                        d[s].unpack(x);
#pragma unroll
                        for (int i = 0; i < 8; ++i) y[i] = decay_gate(x[i] + bb[i], es);
                        st8(p.alpha + g[s], y);
                        e[s].unpack(x);
#pragma unroll
                        for (int i = 0; i < 8; ++i) y[i] = sigmoidf(x[i]);
                        st8(p.erase + g[s], y);
                    }
                }
            }
        }
        {
            const int upr = V / 8, n = nt * upr;
            for (int u0 = tid; u0 < n; u0 += GU * THREADS) {
                Pack8<TI> w[GU];
                size_t g[GU];
#pragma unroll
                for (int s = 0; s < GU; ++s) {
                    const int u = u0 + s * THREADS;
                    if (u < n) {
                        const int r = u / upr, j = u - r * upr;
                        g[s] = ((size_t)b * T + t0 + r) * HV + (size_t)h * V + 8 * j;
                        w[s].load(pw + g[s]);
                    }
                }
#pragma unroll
                for (int s = 0; s < GU; ++s) {
                    if (u0 + s * THREADS < n) {
                        float x[8], y[8];
                        w[s].unpack(x);
#pragma unroll
                        for (int i = 0; i < 8; ++i) y[i] = sigmoidf(x[i]);
                        st8(p.write + g[s], y);
                    }
                }
            }
        }
    } else {
        for (int x = tid; x < nt * K; x += THREADS) {
            const int r = x / K, c = x - r * K;
            const size_t g = ((size_t)b * T + t0 + r) * HK + (size_t)h * K + c;
            const float dz = to_f32(pd[g]), ez = to_f32(pe[g]);
            p.alpha[g] = decay_gate(dz + p.bias[(size_t)h * K + c], es);
            p.erase[g] = sigmoidf(ez);
        }
        for (int x = tid; x < nt * V; x += THREADS) {
            const int r = x / V, c = x - r * V;
            const size_t g = ((size_t)b * T + t0 + r) * HV + (size_t)h * V + c;
            p.write[g] = sigmoidf(to_f32(pw[g]));
        }
    }
    __syncthreads();  // the flags are in shared memory
    // conv masks per token, bit lag: the source is in the destination's document (no valid reset
    // in (source, dest]) and both tokens are valid
    unsigned* smask = reinterpret_cast<unsigned*>(smraw + L.mask);
    for (int r = tid; r < TT; r += THREADS) {
        const int t = t0 + r, rr = r + W - 1;
        unsigned bits = 0;
        bool same_doc = true;
        for (int lag = 0; lag < W; ++lag) {
            if (lag > 0 && same_doc) same_doc = !(sr[rr - lag + 1] != 0.f && sv[rr - lag + 1] != 0.f);
            if (t - lag >= 0 && sv[rr] != 0.f && same_doc && sv[rr - lag] != 0.f) bits |= 1u << lag;
        }
        smask[r] = bits;
    }
    if constexpr (VEC) cp_async_wait_all();
    __syncthreads();

    // 3. q, k, v: one warp per token of the tile
    for (int r = warp; r < nt; r += THREADS / 32) {
        const int t = t0 + r;
        const int rr = r + W - 1;  // the token's staged row
        const unsigned mk = smask[r];
        const size_t gk = ((size_t)b * T + t) * HK + (size_t)h * K, gv = ((size_t)b * T + t) * HV + (size_t)h * V;
        conv_row<TI, TO, E, WT, true>(xq, wq, K, W, rr, mk, lane, static_cast<TO*>(p.q) + gk);
        conv_row<TI, TO, E, WT, true>(xk, wk, K, W, rr, mk, lane, static_cast<TO*>(p.k) + gk);
        conv_row<TI, TO, E, WT, false>(xv, wv, V, W, rr, mk, lane, static_cast<TO*>(p.v) + gv);
    }
}

bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

template <typename TI, typename TO, bool VEC, int WT, int CT = 0>
cudaError_t launch_v(const ProParams& p, cudaStream_t st) {
    const size_t smem = layout(p.K, p.V, p.W, (int)sizeof(TI)).total;
    if (smem > 48 * 1024) {
        const cudaError_t e = cudaFuncSetAttribute(prologue_kernel<TI, TO, VEC, WT, CT>,
                                                   cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    const size_t tiles = (size_t)(p.T + TT - 1) / TT;
    prologue_kernel<TI, TO, VEC, WT, CT><<<(unsigned)(tiles * p.B * p.H), THREADS, smem, st>>>(p);
    return cudaGetLastError();
}

template <typename TI, typename TO>
cudaError_t launch(const ProParams& p, cudaStream_t st) {
    const bool vec = p.K % 8 == 0 && p.V % 8 == 0 && aligned16(p.pq) && aligned16(p.pk) && aligned16(p.pv) &&
                     aligned16(p.pd) && aligned16(p.pe) && aligned16(p.pw) && aligned16(p.cq) && aligned16(p.ck) &&
                     aligned16(p.cv) && aligned16(p.bias) && aligned16(p.q) && aligned16(p.k) && aligned16(p.v) &&
                     aligned16(p.alpha) && aligned16(p.erase) && aligned16(p.write);
    if (!vec) return launch_v<TI, TO, false, 0>(p, st);
    if (p.W == 4 && p.K == 128 && p.V == 128) return launch_v<TI, TO, true, 4, 128>(p, st);
    return p.W == 4 ? launch_v<TI, TO, true, 4>(p, st) : launch_v<TI, TO, true, 0>(p, st);
}

}  // namespace
}  // namespace dbl

extern "C" int dbl_gdn2_prologue(const dbl_gdn2_prologue_args* a, dbl_stream_t stream) {
    using namespace dbl;
    if (!a) return fail(DBL_ERR_INVALID_ARGUMENT, "gdn2_prologue: null args");
    if (a->batch <= 0 || a->time <= 0 || a->heads <= 0 || a->key_dim <= 0 || a->value_dim <= 0)
        return fail(DBL_ERR_INVALID_ARGUMENT, "GDN-2 requires nonempty axes");
    if (a->conv_width < 1 || a->conv_width > MAXW)
        return fail(DBL_ERR_UNSUPPORTED, "gdn2_prologue: convolution width must be 1..=8");
    if (a->key_dim > MAXC || a->value_dim > MAXC)
        return fail(DBL_ERR_UNSUPPORTED, "gdn2_prologue: key and value widths up to 256");
    if ((a->in_dtype != DBL_F32 && a->in_dtype != DBL_BF16) || (a->out_dtype != DBL_F32 && a->out_dtype != DBL_BF16))
        return fail(DBL_ERR_INVALID_ARGUMENT, "gdn2_prologue: dtypes must be f32 or bf16");
    if (!a->proj_q || !a->proj_k || !a->proj_v || !a->proj_decay || !a->proj_erase || !a->proj_write || !a->conv_q ||
        !a->conv_k || !a->conv_v || !a->decay_bias || !a->decay_scale || !a->valid || !a->reset || !a->q || !a->k ||
        !a->v || !a->alpha || !a->erase || !a->write)
        return fail(DBL_ERR_INVALID_ARGUMENT, "gdn2_prologue: every pointer is required");
    if (a->batch * a->time * a->heads > 0x7fffffffLL * 8 || a->time > 0x7fffffff || a->heads > 0x7fffffff)
        return fail(DBL_ERR_UNSUPPORTED, "GDN-2 axis exceeds 32-bit limits");
    ProParams p{};
    p.B = (int)a->batch;
    p.T = (int)a->time;
    p.H = (int)a->heads;
    p.K = (int)a->key_dim;
    p.V = (int)a->value_dim;
    p.W = (int)a->conv_width;
    p.pq = a->proj_q;
    p.pk = a->proj_k;
    p.pv = a->proj_v;
    p.pd = a->proj_decay;
    p.pe = a->proj_erase;
    p.pw = a->proj_write;
    p.cq = a->conv_q;
    p.ck = a->conv_k;
    p.cv = a->conv_v;
    p.bias = a->decay_bias;
    p.scale = a->decay_scale;
    p.valid = a->valid;
    p.reset = a->reset;
    p.q = a->q;
    p.k = a->k;
    p.v = a->v;
    p.alpha = a->alpha;
    p.erase = a->erase;
    p.write = a->write;
    if (a->batch * a->heads * ((a->time + TT - 1) / TT) > 0x7fffffffLL)
        return fail(DBL_ERR_UNSUPPORTED, "gdn2_prologue: grid exceeds 32-bit limits");
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const bool in16 = a->in_dtype == DBL_BF16, out16 = a->out_dtype == DBL_BF16;
    cudaError_t e;
    if (in16 && out16) e = launch<__nv_bfloat16, __nv_bfloat16>(p, st);
    else if (in16) e = launch<__nv_bfloat16, float>(p, st);
    else if (out16) e = launch<float, __nv_bfloat16>(p, st);
    else e = launch<float, float>(p, st);
    return e == cudaSuccess ? DBL_OK : cuda_status(e, "gdn2_prologue launch");
}
