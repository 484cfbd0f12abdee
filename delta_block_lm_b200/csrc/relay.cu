// Relay attention, decode case: split softmax over a shared prefix KV and
// each sequence's own KV, merged by log-sum-exp inside ONE kernel launch.
//
// Arithmetic follows relay_attention_kernel.rs:63-128 (reuse/crates/dre-attention): scores
// q.k * scale, a running maximum, sum of exp(score - max), output acc / sum, and the
// statistics [max, sum] per query; a query with no eligible key writes o = 0, [0, 1].
//
// Work split (one grid, 256 threads per CTA):
//   prefix CTAs (head h, prefix block pb): read the block's keys/values of head h ONCE and
//       produce partials (max, sum, acc[D]) for the queries of EVERY sequence at head h, so the
//       shared prefix is read once per head, never once per sequence.  bf16 inputs stream 512
//       keys per CTA through tensor-core tiles (mma.sync m16n8k16, online softmax over 32-key
//       sub-tiles; 8 warps = 4 query blocks x 2 output halves); f32 inputs use SIMT tiles of 64
//       keys (two partials per CTA).
//   own CTAs (sequence n, head h, 1024-key own block ob): one query against up to 1024 keys,
//       streamed with 16-byte coalesced loads.  bf16: a single pass per warp with an online
//       softmax, K and V rows of a key group loaded together (HBM-bound); f32: scores, then
//       values, with the prefix path's exact arithmetic.
// Each CTA writes its partials to the workspace and bumps a per-(n, h) arrival counter; the
// CTA that completes a row merges its P partials (max of partial maxima, rescaled sums) and
// writes o, max and sum.  The host clears the counters before each launch.
#include <float.h>

#include "common.cuh"

namespace dbl {
namespace {

constexpr int BP = 64;        // prefix keys per tile
constexpr int KSPLIT = 2;     // f32 path: partials per prefix CTA (key halves of 32)
constexpr int TILES_BF16 = 8; // bf16 path: 64-key tiles streamed by one prefix CTA (512 keys)
constexpr int NQ = 64;        // queries per prefix tile
constexpr int BO = 1024;      // own keys per own CTA
constexpr int THREADS = 256;
constexpr int MIN_BLOCKS = 3; // CTAs per SM the register budget is sized for
constexpr int PAD = 8;        // bf16 row padding (row stride D+8 elements: conflict-free ldmatrix)

struct RelayParams {
    int N, H, Lp, Lo, NPB, NOB, P;
    int bpc, ppc;  // prefix keys per prefix CTA, partials per prefix CTA
    float scale;
    const void *q, *kp, *vp, *ko, *vo;
    const int32_t* own_len;
    void* out;
    float *row_max, *row_sum;
    float *part_acc, *part_max, *part_sum;  // [N,H,P,D], [N,H,P], [N,H,P]
    unsigned* counter;                      // [N,H]
};

__device__ __forceinline__ float warp_max(float x) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, o));
    return x;
}
__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
    return x;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void mma_bf16(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
}

// Merges the P partials of row (n, h) and writes the final output and statistics.  The weights
// exp(m_i - M) of the partials are computed once into shared memory (wsm, >= P floats).
template <int D, typename T>
__device__ void merge_row(const RelayParams& p, int n, int h, float* wsm) {
    __shared__ float s_m, s_tot;
    __shared__ int s_any;
    const int tid = threadIdx.x;
    const size_t row = (size_t)n * p.H + h;
    const float* pm = p.part_max + row * p.P;
    const float* ps = p.part_sum + row * p.P;
    if (tid < 32) {
        float m = -FLT_MAX;
        int any = 0;
        for (int i = tid; i < p.P; i += 32)
            if (__ldcg(ps + i) > 0.f) {
                m = fmaxf(m, __ldcg(pm + i));
                any = 1;
            }
        m = warp_max(m);
        any = __any_sync(0xffffffffu, any);
        float tot = 0.f;
        for (int i = tid; i < p.P; i += 32) {
            const float si = __ldcg(ps + i);
            const float w = si > 0.f ? __expf(__ldcg(pm + i) - m) : 0.f;
            wsm[i] = w;
            tot += si * w;
        }
        tot = warp_sum(tot);
        if (tid == 0) {
            s_m = m;
            s_tot = tot;
            s_any = any;
        }
    }
    __syncthreads();
    T* out = static_cast<T*>(p.out) + row * D;
    if (!s_any) {
        for (int d = tid; d < D; d += THREADS) out[d] = from_f32<T>(0.f);
        if (tid == 0) {
            if (p.row_max) p.row_max[row] = 0.f;
            if (p.row_sum) p.row_sum[row] = 1.f;
        }
    } else {
        const float* pa = p.part_acc + row * p.P * D;
        const float inv = 1.f / s_tot;
        for (int d = tid; d < D; d += THREADS) {
            float acc = 0.f;
            for (int i = 0; i < p.P; ++i) acc = fmaf(wsm[i], __ldcg(pa + (size_t)i * D + d), acc);
            out[d] = from_f32<T>(acc * inv);
        }
        if (tid == 0) {
            if (p.row_max) p.row_max[row] = s_m;
            if (p.row_sum) p.row_sum[row] = s_tot;
        }
    }
    __syncthreads();
}

// Adds `inc` arrivals to rows (n0 + r, h), r < nq, and merges the rows this CTA completed.
template <int D, typename T>
__device__ void arrive_rows(const RelayParams& p, int n0, int nq, int h, unsigned inc, float* wsm) {
    __shared__ int s_last[NQ];
    __shared__ int s_nlast;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_nlast = 0;
    __syncthreads();
    if ((int)threadIdx.x < nq) {
        const unsigned prev = atomicAdd(p.counter + (size_t)(n0 + threadIdx.x) * p.H + h, inc);
        if (prev + inc == (unsigned)p.P) s_last[atomicAdd(&s_nlast, 1)] = n0 + threadIdx.x;
    }
    __syncthreads();
    const int nl = s_nlast;
    if (nl > 0) {
        __threadfence();
        for (int i = 0; i < nl; ++i) {
            merge_row<D, T>(p, s_last[i], h, wsm);
            if (threadIdx.x == 0) p.counter[(size_t)s_last[i] * p.H + h] = 0u;
        }
    }
    __syncthreads();
}

// ------------------------------------------------------------------ prefix partials, bf16 MMA
// A prefix CTA streams up to TILES_BF16 x 64 keys of head h through shared memory and keeps, per
// query, an online-softmax partial (max, sum, acc[D]) -- the relay_attention_kernel.rs:73-111
// recurrence, applied to 32-key sub-tiles of tensor-core scores.  Warp w owns queries
// [16 (w & 3), +16) and output dimensions [D/2 (w >> 2), +D/2); both warps of a query block
// compute the same scores.
template <int D>
__device__ void prefix_block_bf16(const RelayParams& p, unsigned char* smem) {
    using T = __nv_bfloat16;
    constexpr int LD = D + PAD;
    constexpr int DH = D / 2;  // output dims per warp
    T* sQ = reinterpret_cast<T*>(smem);  // [NQ][LD]
    T* sK = sQ + NQ * LD;                // [BP][LD]
    T* sV = sK + BP * LD;                // [BP][LD]
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int h = blockIdx.x / p.NPB, pb = blockIdx.x - h * p.NPB;
    const int qb = warp & 3, dh = warp >> 2;
    const int keyA = pb * p.bpc;
    const int keyB = min(p.Lp, keyA + p.bpc);
    constexpr int CPR = D / 8;  // 16-byte chunks per row
    for (int n0 = 0; n0 < p.N; n0 += NQ) {
        const int nq = min(NQ, p.N - n0);
        __syncthreads();
        for (int x = tid; x < NQ * CPR; x += THREADS) {
            const int r = x / CPR, c = (x - r * CPR) * 8;
            uint4 qv = make_uint4(0, 0, 0, 0);
            if (r < nq) qv = *reinterpret_cast<const uint4*>(static_cast<const T*>(p.q) + ((size_t)(n0 + r) * p.H + h) * D + c);
            *reinterpret_cast<uint4*>(sQ + r * LD + c) = qv;
        }
        float m0 = -FLT_MAX, m1 = -FLT_MAX, l0 = 0.f, l1 = 0.f;
        float o[DH / 8][4];
#pragma unroll
        for (int j = 0; j < DH / 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
        for (int k0 = keyA; k0 < keyB; k0 += BP) {
            const int nkeys = min(BP, keyB - k0);
            const T* kp = static_cast<const T*>(p.kp) + ((size_t)h * p.Lp + k0) * D;
            const T* vp = static_cast<const T*>(p.vp) + ((size_t)h * p.Lp + k0) * D;
            __syncthreads();  // previous tile consumed
            for (int x = tid; x < BP * CPR; x += THREADS) {
                const int r = x / CPR, c = (x - r * CPR) * 8;
                uint4 kv = make_uint4(0, 0, 0, 0), vv = make_uint4(0, 0, 0, 0);
                if (r < nkeys) {
                    kv = __ldcs(reinterpret_cast<const uint4*>(kp + (size_t)r * D + c));
                    vv = __ldcs(reinterpret_cast<const uint4*>(vp + (size_t)r * D + c));
                }
                *reinterpret_cast<uint4*>(sK + r * LD + c) = kv;
                *reinterpret_cast<uint4*>(sV + r * LD + c) = vv;
            }
            __syncthreads();
#pragma unroll 1
            for (int sub = 0; sub < BP; sub += 32) {
                // S[16 x 32] = Q[qb] K[sub..sub+32]^T
                float sc[4][4];
#pragma unroll
                for (int j = 0; j < 4; ++j) sc[j][0] = sc[j][1] = sc[j][2] = sc[j][3] = 0.f;
#pragma unroll
                for (int kk = 0; kk < D; kk += 16) {
                    uint32_t a0, a1, a2, a3;
                    ldsm_x4(smem_u32(sQ + (qb * 16 + (lane & 7) + ((lane >> 3) & 1) * 8) * LD + kk + (lane >> 4) * 8), a0, a1, a2,
                            a3);
#pragma unroll
                    for (int nt = 0; nt < 4; nt += 2) {
                        uint32_t b0, b1, b2, b3;
                        ldsm_x4(smem_u32(sK + (sub + nt * 8 + (lane & 7) + (lane >> 4) * 8) * LD + kk + ((lane >> 3) & 1) * 8), b0,
                                b1, b2, b3);
                        mma_bf16(sc[nt], a0, a1, a2, a3, b0, b1);
                        mma_bf16(sc[nt + 1], a0, a1, a2, a3, b2, b3);
                    }
                }
                float t0 = -FLT_MAX, t1 = -FLT_MAX;
#pragma unroll
                for (int nt = 0; nt < 4; ++nt)
#pragma unroll
                    for (int e = 0; e < 2; ++e) {
                        const bool ok = sub + nt * 8 + (lane & 3) * 2 + e < nkeys;
                        sc[nt][e] = ok ? sc[nt][e] * p.scale : -FLT_MAX;
                        sc[nt][2 + e] = ok ? sc[nt][2 + e] * p.scale : -FLT_MAX;
                        t0 = fmaxf(t0, sc[nt][e]);
                        t1 = fmaxf(t1, sc[nt][2 + e]);
                    }
                t0 = fmaxf(t0, __shfl_xor_sync(0xffffffffu, t0, 1));
                t0 = fmaxf(t0, __shfl_xor_sync(0xffffffffu, t0, 2));
                t1 = fmaxf(t1, __shfl_xor_sync(0xffffffffu, t1, 1));
                t1 = fmaxf(t1, __shfl_xor_sync(0xffffffffu, t1, 2));
                if (sub >= nkeys) continue;  // no key in this sub-tile
                const float n0m = fmaxf(m0, t0), n1m = fmaxf(m1, t1);
                const float c0 = l0 > 0.f ? __expf(m0 - n0m) : 0.f, c1 = l1 > 0.f ? __expf(m1 - n1m) : 0.f;
                m0 = n0m;
                m1 = n1m;
                float s0 = 0.f, s1 = 0.f;
                uint32_t pa[2][4];
#pragma unroll
                for (int nt = 0; nt < 4; ++nt) {
                    float e0[2], e1[2];
#pragma unroll
                    for (int e = 0; e < 2; ++e) {
                        const bool ok = sub + nt * 8 + (lane & 3) * 2 + e < nkeys;
                        e0[e] = ok ? __expf(sc[nt][e] - m0) : 0.f;
                        e1[e] = ok ? __expf(sc[nt][2 + e] - m1) : 0.f;
                        s0 += e0[e];
                        s1 += e1[e];
                    }
                    const int ks = nt >> 1, hi = nt & 1;
                    pa[ks][hi ? 2 : 0] = pack_bf16(e0[0], e0[1]);
                    pa[ks][hi ? 3 : 1] = pack_bf16(e1[0], e1[1]);
                }
                s0 += __shfl_xor_sync(0xffffffffu, s0, 1);
                s0 += __shfl_xor_sync(0xffffffffu, s0, 2);
                s1 += __shfl_xor_sync(0xffffffffu, s1, 1);
                s1 += __shfl_xor_sync(0xffffffffu, s1, 2);
                l0 = l0 * c0 + s0;
                l1 = l1 * c1 + s1;
#pragma unroll
                for (int j = 0; j < DH / 8; ++j) {
                    o[j][0] *= c0;
                    o[j][1] *= c0;
                    o[j][2] *= c1;
                    o[j][3] *= c1;
                }
                // O[16 x DH] += P[16 x 32] V[sub..sub+32][dh*DH ..]
#pragma unroll
                for (int ks = 0; ks < 2; ++ks) {
#pragma unroll
                    for (int dt = 0; dt < DH / 8; dt += 2) {
                        uint32_t b0, b1, b2, b3;
                        ldsm_x4_t(smem_u32(sV + (sub + ks * 16 + (lane & 7) + ((lane >> 3) & 1) * 8) * LD + dh * DH + dt * 8 +
                                           (lane >> 4) * 8),
                                  b0, b1, b2, b3);
                        mma_bf16(o[dt], pa[ks][0], pa[ks][1], pa[ks][2], pa[ks][3], b0, b1);
                        mma_bf16(o[dt + 1], pa[ks][0], pa[ks][1], pa[ks][2], pa[ks][3], b2, b3);
                    }
                }
            }
        }
        const int pidx = pb;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
            const int r = qb * 16 + (lane >> 2) + half * 8;
            if (r < nq) {
                const size_t row = (size_t)(n0 + r) * p.H + h;
                float* dst = p.part_acc + (row * p.P + pidx) * D + dh * DH;
#pragma unroll
                for (int dt = 0; dt < DH / 8; ++dt)
                    *reinterpret_cast<float2*>(dst + dt * 8 + (lane & 3) * 2) = make_float2(o[dt][half * 2], o[dt][half * 2 + 1]);
                if (dh == 0 && (lane & 3) == 0) {
                    p.part_max[row * p.P + pidx] = half ? m1 : m0;
                    p.part_sum[row * p.P + pidx] = half ? l1 : l0;
                }
            }
        }
        arrive_rows<D, T>(p, n0, nq, h, 1u, reinterpret_cast<float*>(smem));
    }
}

// ------------------------------------------------------------------ prefix partials, f32 SIMT
template <int D>
__device__ void prefix_block_f32(const RelayParams& p, unsigned char* smem) {
    constexpr int HK = BP / KSPLIT;  // 32 keys per half
    constexpr int QT = 32;           // queries per inner tile
    float* sK = reinterpret_cast<float*>(smem);  // [HK][D+1]
    float* sV = sK + HK * (D + 1);               // [HK][D]
    float* sQ = sV + HK * D;                     // [QT][D+1]
    float* sS = sQ + QT * (D + 1);               // [QT][HK+1]
    const int tid = threadIdx.x;
    const int h = blockIdx.x / p.NPB, pb = blockIdx.x - h * p.NPB;
    for (int kh = 0; kh < KSPLIT; ++kh) {
        const int key0 = pb * BP + kh * HK;
        const int nkeys = max(0, min(HK, p.Lp - key0));
        const float* kp = static_cast<const float*>(p.kp) + ((size_t)h * p.Lp + key0) * D;
        const float* vp = static_cast<const float*>(p.vp) + ((size_t)h * p.Lp + key0) * D;
        __syncthreads();
        for (int x = tid; x < HK * D; x += THREADS) {
            const int r = x / D, c = x - r * D;
            sK[r * (D + 1) + c] = r < nkeys ? kp[x] : 0.f;
            sV[r * D + c] = r < nkeys ? vp[x] : 0.f;
        }
        for (int n0 = 0; n0 < p.N; n0 += QT) {
            const int nq = min(QT, p.N - n0);
            __syncthreads();
            for (int x = tid; x < QT * D; x += THREADS) {
                const int r = x / D, c = x - r * D;
                sQ[r * (D + 1) + c] =
                    r < nq ? static_cast<const float*>(p.q)[((size_t)(n0 + r) * p.H + h) * D + c] * p.scale : 0.f;
            }
            __syncthreads();
            {  // thread: query tid/8, keys (tid%8) + 8b
                const int qi = tid >> 3, kg = tid & 7;
                float acc[4] = {0.f, 0.f, 0.f, 0.f};
                for (int c = 0; c < D; ++c) {
                    const float qv = sQ[qi * (D + 1) + c];
#pragma unroll
                    for (int b = 0; b < 4; ++b) acc[b] = fmaf(qv, sK[(kg + 8 * b) * (D + 1) + c], acc[b]);
                }
#pragma unroll
                for (int b = 0; b < 4; ++b) {
                    const int key = kg + 8 * b;
                    sS[qi * (HK + 1) + key] = key < nkeys ? acc[b] : -FLT_MAX;
                }
            }
            __syncthreads();
            if (tid < QT) {
                const int r = tid;
                float m = -FLT_MAX, l = 0.f;
                for (int c = 0; c < HK; ++c) m = fmaxf(m, sS[r * (HK + 1) + c]);
                for (int c = 0; c < HK; ++c) {
                    const float e = c < nkeys ? __expf(sS[r * (HK + 1) + c] - m) : 0.f;
                    sS[r * (HK + 1) + c] = e;
                    l += e;
                }
                if (r < nq) {
                    const size_t row = (size_t)(n0 + r) * p.H + h;
                    p.part_max[row * p.P + pb * KSPLIT + kh] = m;
                    p.part_sum[row * p.P + pb * KSPLIT + kh] = nkeys > 0 ? l : 0.f;
                }
            }
            __syncthreads();
            {  // thread: query tid/8, dims (tid%8) + 8c
                const int qi = tid >> 3, dg = tid & 7;
                float acc[D / 8];
#pragma unroll
                for (int c = 0; c < D / 8; ++c) acc[c] = 0.f;
                for (int key = 0; key < HK; ++key) {
                    const float e = sS[qi * (HK + 1) + key];
#pragma unroll
                    for (int c = 0; c < D / 8; ++c) acc[c] = fmaf(e, sV[key * D + dg + 8 * c], acc[c]);
                }
                if (qi < nq) {
                    const size_t row = (size_t)(n0 + qi) * p.H + h;
                    float* dst = p.part_acc + (row * p.P + pb * KSPLIT + kh) * D;
#pragma unroll
                    for (int c = 0; c < D / 8; ++c) dst[dg + 8 * c] = acc[c];
                }
            }
        }
    }
    // Both partials of every row are written: KSPLIT arrivals per row.
    for (int n0 = 0; n0 < p.N; n0 += NQ) arrive_rows<D, float>(p, n0, min(NQ, p.N - n0), h, KSPLIT, reinterpret_cast<float*>(smem));
}

// ------------------------------------------------------------------------- own-segment partials
template <int D, typename T>
__device__ void own_block(const RelayParams& p, unsigned char* smem) {
    constexpr int EPL = 16 / sizeof(T);   // elements per 16-byte lane load
    constexpr int LPK = D / EPL;          // lanes per key row
    constexpr int KPW = 32 / LPK;         // keys per warp instruction
    constexpr int NW = THREADS / 32;
    float* se = reinterpret_cast<float*>(smem);  // [BO]
    float* sacc = se + BO;                       // [NW][D]
    __shared__ float s_red[2][NW];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int bid = blockIdx.x - p.H * p.NPB;
    const int ob = bid % p.NOB;
    const int nh = bid / p.NOB;
    const int n = nh / p.H, h = nh - n * p.H;
    const int own = p.own_len ? min(max(p.own_len[n], 0), p.Lo) : p.Lo;
    const int key0 = ob * BO;
    const int nkeys = max(0, min(BO, own - key0));
    const size_t row = (size_t)n * p.H + h;
    const int sub = lane / LPK, part = lane % LPK;  // key slot within the warp, chunk of the row
    const T* ko = static_cast<const T*>(p.ko) + (row * p.Lo + key0) * D;
    const T* vo = static_cast<const T*>(p.vo) + (row * p.Lo + key0) * D;
    constexpr int KEYS_PER_WARP = BO / NW;
    constexpr int ITER = KEYS_PER_WARP / KPW;
    if constexpr (sizeof(T) == 4) {
        // f32: the prefix SIMT path's exact arithmetic (pre-scaled q, one fma chain over d), so
        // that equal keys in the two segments give bit-equal scores (relay_tests.rs:47-90).
        float* sq = sacc;  // [D], reused before the value pass
        for (int c = tid; c < D; c += THREADS) sq[c] = to_f32(static_cast<const T*>(p.q)[row * D + c]) * p.scale;
        __syncthreads();
        for (int key = tid; key < BO; key += THREADS) {
            float d = 0.f;
            if (key < nkeys) {
                const T* kr = ko + (size_t)key * D;
#pragma unroll 8
                for (int c = 0; c < D; ++c) d = fmaf(sq[c], to_f32(kr[c]), d);
            }
            se[key] = key < nkeys ? d : -FLT_MAX;
        }
        __syncthreads();
        float m = -FLT_MAX;
        for (int k = lane; k < BO; k += 32) m = fmaxf(m, se[k]);
        m = warp_max(m);  // every warp computes the block max redundantly
        __syncthreads();
        float lsum = 0.f;
        for (int k = tid; k < BO; k += THREADS) {
            const float e = k < nkeys ? __expf(se[k] - m) : 0.f;
            se[k] = e;
            lsum += e;
        }
        lsum = warp_sum(lsum);
        if (lane == 0) s_red[1][warp] = lsum;
        __syncthreads();
        float l = 0.f;
#pragma unroll
        for (int w = 0; w < NW; ++w) l += s_red[1][w];
        // acc[d] = sum_key e[key] v[key][d]; lane holds EPL dims of one key slot
        float acc[EPL];
#pragma unroll
        for (int e = 0; e < EPL; ++e) acc[e] = 0.f;
#pragma unroll 8
        for (int it = 0; it < ITER; ++it) {
            const int key = warp * KEYS_PER_WARP + it * KPW + sub;
            if (key < nkeys) {
                const uint4 raw = __ldcs(reinterpret_cast<const uint4*>(vo + (size_t)key * D + part * EPL));
                const T* x = reinterpret_cast<const T*>(&raw);
                const float w = se[key];
#pragma unroll
                for (int e = 0; e < EPL; ++e) acc[e] = fmaf(w, to_f32(x[e]), acc[e]);
            }
        }
#pragma unroll
        for (int o = LPK; o < 32; o <<= 1)
#pragma unroll
            for (int e = 0; e < EPL; ++e) acc[e] += __shfl_xor_sync(0xffffffffu, acc[e], o);
        if (sub == 0)
#pragma unroll
            for (int e = 0; e < EPL; ++e) sacc[warp * D + part * EPL + e] = acc[e];
        __syncthreads();
        const int pi = p.NPB * p.ppc + ob;
        for (int d = tid; d < D; d += THREADS) {
            float a = 0.f;
#pragma unroll
            for (int w = 0; w < NW; ++w) a += sacc[w * D + d];
            p.part_acc[(row * p.P + pi) * D + d] = a;
        }
        if (tid == 0) {
            p.part_max[row * p.P + pi] = m;
            p.part_sum[row * p.P + pi] = nkeys > 0 ? l : 0.f;
        }
    } else {
        // bf16: one pass.  Each warp runs an online softmax over its keys in groups of KPW x U,
        // loading the K and V rows of a group together (2U 16-byte loads in flight per lane);
        // products of bf16 values are exact in f32 and the score is scaled after the sum, as the
        // tensor-core prefix path does.  The warps' (max, sum, acc) are merged at the end.
        constexpr int U = 4;
        float qv[EPL];
        const T* q = static_cast<const T*>(p.q) + row * D + part * EPL;
#pragma unroll
        for (int e = 0; e < EPL; ++e) qv[e] = to_f32(q[e]);
        float m = -FLT_MAX, l = 0.f, acc[EPL];
#pragma unroll
        for (int e = 0; e < EPL; ++e) acc[e] = 0.f;
        for (int g = 0; g < ITER; g += U) {
            uint4 kr[U], vr[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int key = warp * KEYS_PER_WARP + (g + u) * KPW + sub;
                if (key < nkeys) {
                    kr[u] = __ldcs(reinterpret_cast<const uint4*>(ko + (size_t)key * D + part * EPL));
                    vr[u] = __ldcs(reinterpret_cast<const uint4*>(vo + (size_t)key * D + part * EPL));
                } else {
                    kr[u] = make_uint4(0, 0, 0, 0);
                    vr[u] = make_uint4(0, 0, 0, 0);
                }
            }
            float sc[U];
            float mg = -FLT_MAX;
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const T* x = reinterpret_cast<const T*>(&kr[u]);
                float d = 0.f;
#pragma unroll
                for (int e = 0; e < EPL; ++e) d = fmaf(qv[e], to_f32(x[e]), d);
#pragma unroll
                for (int o = LPK / 2; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
                const int key = warp * KEYS_PER_WARP + (g + u) * KPW + sub;
                sc[u] = key < nkeys ? d * p.scale : -FLT_MAX;
                mg = fmaxf(mg, sc[u]);
            }
#pragma unroll
            for (int o = LPK; o < 32; o <<= 1) mg = fmaxf(mg, __shfl_xor_sync(0xffffffffu, mg, o));  // every key slot
            const float mn = fmaxf(m, mg);
            const float corr = __expf(m - mn);  // 0 while nothing was seen (acc and l are 0 then)
            l *= corr;
#pragma unroll
            for (int e = 0; e < EPL; ++e) acc[e] *= corr;
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int key = warp * KEYS_PER_WARP + (g + u) * KPW + sub;
                const float w = key < nkeys ? __expf(sc[u] - mn) : 0.f;
                if (part == 0) l += w;
                const T* x = reinterpret_cast<const T*>(&vr[u]);
#pragma unroll
                for (int e = 0; e < EPL; ++e) acc[e] = fmaf(w, to_f32(x[e]), acc[e]);
            }
            m = mn;
        }
#pragma unroll
        for (int o = LPK; o < 32; o <<= 1)
#pragma unroll
            for (int e = 0; e < EPL; ++e) acc[e] += __shfl_xor_sync(0xffffffffu, acc[e], o);
        l = warp_sum(l);
        if (sub == 0)
#pragma unroll
            for (int e = 0; e < EPL; ++e) sacc[warp * D + part * EPL + e] = acc[e];
        if (lane == 0) {
            s_red[0][warp] = m;
            s_red[1][warp] = l;
        }
        __syncthreads();
        float mb = -FLT_MAX;
#pragma unroll
        for (int w = 0; w < NW; ++w) mb = fmaxf(mb, s_red[0][w]);
        float fw[NW], lb = 0.f;
#pragma unroll
        for (int w = 0; w < NW; ++w) {
            fw[w] = __expf(s_red[0][w] - mb);
            lb = fmaf(fw[w], s_red[1][w], lb);
        }
        const int pi = p.NPB * p.ppc + ob;
        for (int d = tid; d < D; d += THREADS) {
            float a = 0.f;
#pragma unroll
            for (int w = 0; w < NW; ++w) a = fmaf(fw[w], sacc[w * D + d], a);
            p.part_acc[(row * p.P + pi) * D + d] = a;
        }
        if (tid == 0) {
            p.part_max[row * p.P + pi] = mb;
            p.part_sum[row * p.P + pi] = nkeys > 0 ? lb : 0.f;
        }
    }
    arrive_rows<D, T>(p, n, 1, h, 1u, se);
}

template <int D, typename T>
__global__ void __launch_bounds__(THREADS, MIN_BLOCKS) relay_merge_kernel(const RelayParams p) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    if ((int)blockIdx.x < p.H * p.NPB) {
        if constexpr (sizeof(T) == 2) prefix_block_bf16<D>(p, smem_raw);
        else prefix_block_f32<D>(p, smem_raw);
    } else {
        own_block<D, T>(p, smem_raw);
    }
}

size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

struct Layout {
    int NPB, NOB, P, bpc, ppc;
    size_t off_acc, off_max, off_sum, off_cnt, total;
};

// bf16: one partial per 512-key prefix CTA; f32: two partials per 64-key prefix CTA.
Layout layout(int64_t N, int64_t H, int64_t D, int64_t Lp, int64_t Lo, bool bf16) {
    Layout L{};
    L.bpc = bf16 ? BP * TILES_BF16 : BP;
    L.ppc = bf16 ? 1 : KSPLIT;
    L.NPB = (int)((Lp + L.bpc - 1) / L.bpc);
    L.NOB = (int)((Lo + BO - 1) / BO);
    if (L.NOB == 0) L.NOB = 1;  // one (empty) own partial keeps the arrival count uniform
    L.P = L.NPB * L.ppc + L.NOB;
    const size_t rows = (size_t)N * H;
    L.off_acc = 0;
    L.off_max = align_up(L.off_acc + rows * L.P * D * sizeof(float), 256);
    L.off_sum = align_up(L.off_max + rows * L.P * sizeof(float), 256);
    L.off_cnt = align_up(L.off_sum + rows * L.P * sizeof(float), 256);
    L.total = align_up(L.off_cnt + rows * sizeof(unsigned), 256);
    return L;
}

template <int D, typename T>
size_t relay_smem(int P) {
    size_t prefix;
    if (sizeof(T) == 2) prefix = sizeof(__nv_bfloat16) * (size_t)(NQ + 2 * BP) * (D + PAD);
    else prefix = sizeof(float) * (size_t)((BP / KSPLIT) * (D + 1) + (BP / KSPLIT) * D + 32 * (D + 1) + 32 * (BP / KSPLIT + 1));
    size_t own = sizeof(float) * (size_t)(BO + (THREADS / 32) * D);
    if (own < sizeof(float) * (size_t)P) own = sizeof(float) * (size_t)P;  // merge weights
    if (prefix < sizeof(float) * (size_t)P) prefix = sizeof(float) * (size_t)P;
    return prefix > own ? prefix : own;
}

template <int D, typename T>
int launch_relay(const RelayParams& p, cudaStream_t st) {
    const size_t smem = relay_smem<D, T>(p.P);
    cudaError_t e = cudaFuncSetAttribute(relay_merge_kernel<D, T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return cuda_status(e, "relay: cudaFuncSetAttribute");
    const unsigned grid = (unsigned)(p.H * p.NPB + p.N * p.H * p.NOB);
    relay_merge_kernel<D, T><<<grid, THREADS, smem, st>>>(p);
    return launch_status("relay_merge_kernel");
}

}  // namespace

// Shared by the workspace entry point and any variant that supplies its own scratch.
int relay_validate(const dbl_relay_merge_args* a) {
    if (!a) return fail(DBL_ERR_INVALID_ARGUMENT, "relay: null args");
    if (a->n_seq <= 0 || a->heads <= 0) return fail(DBL_ERR_INVALID_ARGUMENT, "relay: n_seq and heads must be positive");
    if (a->prefix_len < 0 || a->own_cap < 0) return fail(DBL_ERR_INVALID_ARGUMENT, "relay: negative segment length");
    if (a->head_dim != 64 && a->head_dim != 128)
        return fail(DBL_ERR_UNSUPPORTED, "relay: head_dim must be 64 or 128 (got %lld)", (long long)a->head_dim);
    if (a->dtype != DBL_F32 && a->dtype != DBL_BF16) return fail(DBL_ERR_INVALID_ARGUMENT, "relay: dtype must be f32 or bf16");
    if (!a->q || !a->out) return fail(DBL_ERR_INVALID_ARGUMENT, "relay: q and out are required");
    if (a->prefix_len > 0 && (!a->prefix_k || !a->prefix_v))
        return fail(DBL_ERR_INVALID_ARGUMENT, "relay: prefix_k and prefix_v are required when prefix_len > 0");
    if (a->own_cap > 0 && (!a->own_k || !a->own_v))
        return fail(DBL_ERR_INVALID_ARGUMENT, "relay: own_k and own_v are required when own_cap > 0");
    const void* ptrs[5] = {a->q, a->prefix_k, a->prefix_v, a->own_k, a->own_v};
    for (const void* ptr : ptrs)
        if (ptr && !aligned(ptr, 16)) return fail(DBL_ERR_INVALID_ARGUMENT, "relay: q, k and v must be 16-byte aligned");
    if (a->prefix_len > 0x7fffffff || a->own_cap > 0x7fffffff || a->n_seq * a->heads > 0x7fffffff)
        return fail(DBL_ERR_UNSUPPORTED, "relay: sizes exceed 32-bit limits");
    const Layout L = layout(a->n_seq, a->heads, a->head_dim, a->prefix_len, a->own_cap, a->dtype == DBL_BF16);
    const int64_t grid = a->heads * (int64_t)L.NPB + a->n_seq * a->heads * (int64_t)L.NOB;
    if (grid > 0x7fffffffLL) return fail(DBL_ERR_UNSUPPORTED, "relay: grid too large");
    return DBL_OK;
}

// Workspace bytes of one call with the layout of its own dtype.
size_t relay_call_workspace_bytes(const dbl_relay_merge_args* a) {
    return layout(a->n_seq, a->heads, a->head_dim, a->prefix_len, a->own_cap, a->dtype == DBL_BF16).total;
}

size_t relay_workspace_bytes(int64_t N, int64_t H, int64_t D, int64_t Lp, int64_t Lo) {
    // the f32 layout has more prefix partials; it bounds both dtypes
    const size_t a = layout(N, H, D, Lp, Lo, false).total, b = layout(N, H, D, Lp, Lo, true).total;
    return a > b ? a : b;
}

// Launches the merge with its partials placed in `ws`, which must hold at least
// relay_call_workspace_bytes(a) bytes (the layout of the call's own dtype).  The arrival counters
// are cleared first on the same stream.
int relay_launch(const dbl_relay_merge_args* a, void* ws, cudaStream_t st) {
    const Layout L = layout(a->n_seq, a->heads, a->head_dim, a->prefix_len, a->own_cap, a->dtype == DBL_BF16);
    RelayParams p{};
    p.N = (int)a->n_seq;
    p.H = (int)a->heads;
    p.Lp = (int)a->prefix_len;
    p.Lo = (int)a->own_cap;
    p.NPB = L.NPB;
    p.NOB = L.NOB;
    p.P = L.P;
    p.bpc = L.bpc;
    p.ppc = L.ppc;
    p.scale = a->scale;
    p.q = a->q;
    p.kp = a->prefix_k;
    p.vp = a->prefix_v;
    p.ko = a->own_k;
    p.vo = a->own_v;
    p.own_len = a->own_len;
    p.out = a->out;
    p.row_max = a->row_max;
    p.row_sum = a->row_sum;
    unsigned char* base = static_cast<unsigned char*>(ws);
    p.part_acc = reinterpret_cast<float*>(base + L.off_acc);
    p.part_max = reinterpret_cast<float*>(base + L.off_max);
    p.part_sum = reinterpret_cast<float*>(base + L.off_sum);
    p.counter = reinterpret_cast<unsigned*>(base + L.off_cnt);
    cudaError_t e = cudaMemsetAsync(p.counter, 0, sizeof(unsigned) * (size_t)p.N * p.H, st);
    if (e != cudaSuccess) return cuda_status(e, "relay: clear counters");
    const bool bf = a->dtype == DBL_BF16;
    if (a->head_dim == 128) return bf ? launch_relay<128, __nv_bfloat16>(p, st) : launch_relay<128, float>(p, st);
    return bf ? launch_relay<64, __nv_bfloat16>(p, st) : launch_relay<64, float>(p, st);
}

}  // namespace dbl

extern "C" size_t dbl_relay_merge_workspace_bytes(int64_t n_seq, int64_t heads, int64_t head_dim, int64_t prefix_len,
                                                  int64_t own_cap) {
    if (n_seq <= 0 || heads <= 0 || head_dim <= 0 || prefix_len < 0 || own_cap < 0) return 0;
    return dbl::relay_workspace_bytes(n_seq, heads, head_dim, prefix_len, own_cap);
}

extern "C" size_t dbl_relay_merge_call_workspace_bytes(const dbl_relay_merge_args* a) {
    if (!a || a->n_seq <= 0 || a->heads <= 0 || a->head_dim <= 0 || a->prefix_len < 0 || a->own_cap < 0) return 0;
    return dbl::relay_call_workspace_bytes(a);
}

extern "C" int dbl_relay_merge_decode(const dbl_relay_merge_args* a, void* workspace, size_t workspace_bytes,
                                      dbl_stream_t stream) {
    using namespace dbl;
    int rc = relay_validate(a);
    if (rc != DBL_OK) return rc;
    const size_t need = relay_workspace_bytes(a->n_seq, a->heads, a->head_dim, a->prefix_len, a->own_cap);
    if (!workspace || workspace_bytes < need)
        return fail(DBL_ERR_WORKSPACE, "relay: workspace of %zu bytes required (got %zu)", need, workspace_bytes);
    if (!aligned(workspace, 16)) return fail(DBL_ERR_INVALID_ARGUMENT, "relay: workspace must be 16-byte aligned");
    return relay_launch(a, workspace, reinterpret_cast<cudaStream_t>(stream));
}
