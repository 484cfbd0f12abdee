// Relay attention, decode case: split softmax over a shared prefix KV and
// each sequence's own KV, merged by log-sum-exp inside ONE kernel launch.
//
// Arithmetic follows relay_attention_kernel.rs:63-128 (reuse/crates/dre-attention): scores
// q.k * scale, a running maximum, sum of exp(score - max), output acc / sum, and the
// statistics [max, sum] per query; a query with no eligible key writes o = 0, [0, 1].
//
// One CTA (256 threads) per work item:
//   prefix items (head h, prefix block pb): read the block's keys/values of head h ONCE and
//       produce partials (max, sum, acc[D]) for the queries of EVERY sequence at head h, so the
//       shared prefix is read once per head, never once per sequence.  bf16 streams 1024 keys
//       through tensor-core tiles (mma.sync m16n8k16, online softmax over 32-key sub-tiles, two
//       tile buffers); f32 uses SIMT tiles of 64 keys (two partials per item).
//   own items (sequence n, head h, 1024-key own block ob): one query against the block's keys.
//       bf16: streamed through a bulk-copy ring (below); f32: scores then values with the prefix
//       path's exact arithmetic.
// Each item writes its partial to the workspace and bumps a per-(n, h) arrival counter; the
// block that completes a row merges its P partials (max of partial maxima, rescaled sums) and
// writes o, max and sum.  The host clears the counters before each launch.
#include <float.h>

#include "common.cuh"
#include "tc_ptx.cuh"

namespace dbl {
namespace {

constexpr int BP = 64;        // prefix keys per tile
constexpr int KSPLIT = 2;     // f32 path: partials per prefix CTA (key halves of 32)
constexpr int TILES_BF16 = 16; // bf16 path: 64-key tiles streamed by one prefix item (1024 keys; 512 or 2048 measured slower)
constexpr int NQ = 64;        // queries per prefix pass
constexpr int BO = 1024;      // f32: own keys per own CTA
constexpr int THREADS = 256;
constexpr int MIN_BLOCKS_F32 = 3;  // f32 kernel: CTAs per SM its register budget is sized for
constexpr int PAD = 8;        // bf16 row padding (row stride D+8 elements: conflict-free ldmatrix)
constexpr int PLD = BP + 8;   // row stride of a prefix P tile (64 keys + 8: conflict-free ldmatrix)
constexpr int kRelayWaitFull = 30, kRelayWaitEmpty = 31;  // wait-site codes (dbl_device_error)

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
    int* err;                               // the library's device error word
    int bo;                                 // own keys per own item
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
// The two warps of prefix query block qb (warps qb and qb + 4) meet at named barrier 1 + qb; the
// ids are spelled out so that the kernel reserves five barriers, not all sixteen.
__device__ __forceinline__ void pair_sync(int qb) {
    switch (qb) {
        case 0: asm volatile("bar.sync 1, 64;" ::: "memory"); break;
        case 1: asm volatile("bar.sync 2, 64;" ::: "memory"); break;
        case 2: asm volatile("bar.sync 3, 64;" ::: "memory"); break;
        default: asm volatile("bar.sync 4, 64;" ::: "memory"); break;
    }
}
// 16-byte asynchronous global -> shared copy through L2 only; src_bytes = 0 reads nothing and
// fills the 16 bytes with zeros.
__device__ __forceinline__ void cp16_zfill(void* sdst, const void* gsrc, int src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(sdst)), "l"(gsrc), "r"(src_bytes)
                 : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
// Bulk (non-tensor, no multicast) global -> shared copy of `bytes` (a multiple of 16, both
// addresses 16-byte aligned) completing on `bar` with a transaction count.
__device__ __forceinline__ void bulk_g2s(void* sdst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(sdst)),
                 "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}
// Waits for phase `parity` of `bar` for at most kWaitLimitNs, whatever the block's error word says
// (used to drain copies still in flight before a block leaves after an error).
__device__ __forceinline__ void mbar_drain(uint64_t* bar, uint32_t parity) {
    const uint64_t t0 = globaltimer_ns();
    while (!mbar_try_wait(bar, parity))
        if (globaltimer_ns() - t0 > kWaitLimitNs) return;
}

// Merges the P partials of row (n, h) and writes the final output and statistics; one warp.
// Partial i carries (max m_i, sum s_i, acc_i[D]); with M the largest m_i of the partials with
// s_i > 0, w_i = exp(m_i - M) (0 for an empty partial), o = (sum_i w_i acc_i) / (sum_i w_i s_i).
// Lane l owns dims [l D/32, (l + 1) D/32); the weights of 32 partials at a time are held one per
// lane and broadcast.
template <int D, typename T>
__device__ void merge_row(const RelayParams& p, int n, int h, int lane) {
    constexpr int DPL = D / 32;  // dims per lane
    const size_t row = (size_t)n * p.H + h;
    const float* pm = p.part_max + row * p.P;
    const float* ps = p.part_sum + row * p.P;
    float m = -FLT_MAX;
    int any = 0;
    for (int i = lane; i < p.P; i += 32)
        if (__ldcg(ps + i) > 0.f) {
            m = fmaxf(m, __ldcg(pm + i));
            any = 1;
        }
    m = warp_max(m);
    any = __any_sync(0xffffffffu, any);
    T* out = static_cast<T*>(p.out) + row * D + lane * DPL;
    if (!any) {
#pragma unroll
        for (int d = 0; d < DPL; ++d) out[d] = from_f32<T>(0.f);
        if (lane == 0) {
            if (p.row_max) p.row_max[row] = 0.f;
            if (p.row_sum) p.row_sum[row] = 1.f;
        }
        return;
    }
    const float* pa = p.part_acc + row * p.P * D + lane * DPL;
    float acc[DPL], tot = 0.f;
#pragma unroll
    for (int d = 0; d < DPL; ++d) acc[d] = 0.f;
    for (int i0 = 0; i0 < p.P; i0 += 32) {
        const int i = i0 + lane;
        float w = 0.f;
        if (i < p.P) {
            const float si = __ldcg(ps + i);
            w = si > 0.f ? __expf(__ldcg(pm + i) - m) : 0.f;
            tot += si * w;
        }
        const int cnt = min(32, p.P - i0);
#pragma unroll 4
        for (int j = 0; j < cnt; ++j) {
            const float wj = __shfl_sync(0xffffffffu, w, j);
            const float* src = pa + (size_t)(i0 + j) * D;
            if constexpr (DPL == 4) {
                const float4 x = __ldcg(reinterpret_cast<const float4*>(src));
                acc[0] = fmaf(wj, x.x, acc[0]);
                acc[1] = fmaf(wj, x.y, acc[1]);
                acc[2] = fmaf(wj, x.z, acc[2]);
                acc[3] = fmaf(wj, x.w, acc[3]);
            } else {
                const float2 x = __ldcg(reinterpret_cast<const float2*>(src));
                acc[0] = fmaf(wj, x.x, acc[0]);
                acc[1] = fmaf(wj, x.y, acc[1]);
            }
        }
    }
    tot = warp_sum(tot);
    const float inv = 1.f / tot;
#pragma unroll
    for (int d = 0; d < DPL; ++d) out[d] = from_f32<T>(acc[d] * inv);
    if (lane == 0) {
        if (p.row_max) p.row_max[row] = m;
        if (p.row_sum) p.row_sum[row] = tot;
    }
}

// Adds `inc` arrivals to rows (n0 + r, h), r < nq, and merges the rows this CTA completed, one
// warp per row.
template <int D, typename T>
__device__ void arrive_rows(const RelayParams& p, int n0, int nq, int h, unsigned inc) {
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
        const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
        for (int i = warp; i < nl; i += THREADS / 32) {
            merge_row<D, T>(p, s_last[i], h, lane);
            if (lane == 0) p.counter[(size_t)s_last[i] * p.H + h] = 0u;
        }
    }
    __syncthreads();
}

// ------------------------------------------------------------------ prefix partials, bf16 MMA
// A prefix item (head h, prefix block pb) streams up to TILES_BF16 x 64 keys of head h through two
// shared-memory buffers (the next tile in flight while one is computed) and keeps, per query, an
// online-softmax partial (max, sum, acc[D]) -- the relay_attention_kernel.rs:73-111 recurrence,
// applied to 64-key tiles of tensor-core scores (mma.sync: a kernel with tcgen05 instructions runs
// one CTA per SM, which would halve the own stream's residency).  Warp w owns queries
// [16 (w & 3), +16) and output dimensions [D/2 (w >> 2), +D/2); the two warps of a query block
// score one 32-key half of the tile each and exchange their row maxima, row sums and bf16 P
// through shared memory (double-buffered by tile parity, a 64-thread named barrier per pair).
template <int D>
__device__ void prefix_block_bf16(const RelayParams& p, unsigned char* smem, int item) {
    using T = __nv_bfloat16;
    constexpr int LD = D + PAD;
    constexpr int DH = D / 2;  // output dims per warp
    T* sQ = reinterpret_cast<T*>(smem);  // [NQ][LD]
    T* sKb = sQ + NQ * LD;               // [2][BP][LD]: tile t in buffer t & 1
    T* sVb = sKb + 2 * BP * LD;          // [2][BP][LD]
    T* sP = sVb + 2 * BP * LD;           // [2][4][16][PLD]: each query block's P tile, by tile parity
    float* spm = reinterpret_cast<float*>(sP + 2 * 4 * 16 * PLD);  // [2][4][2][16] row maxima per half
    float* sps = spm + 2 * 4 * 2 * 16;                              // [2][4][2][16] row sums per half
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int h = item / p.NPB, pb = item - h * p.NPB;
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
        // K and V tiles stream through two buffers: tile t + 1 is in flight (cp.async, keys past
        // the block's end zero-filled) while tile t is computed.
        auto fetch = [&](int k0, int buf) {
            const int nkeys = min(BP, keyB - k0);
            const T* kp = static_cast<const T*>(p.kp) + ((size_t)h * p.Lp + k0) * D;
            const T* vp = static_cast<const T*>(p.vp) + ((size_t)h * p.Lp + k0) * D;
            T* dK = sKb + buf * BP * LD;
            T* dV = sVb + buf * BP * LD;
            for (int x = tid; x < BP * CPR; x += THREADS) {
                const int r = x / CPR, c = (x - r * CPR) * 8;
                const bool ok = r < nkeys;
                const size_t off = (size_t)(ok ? r : 0) * D + c;
                cp16_zfill(dK + r * LD + c, kp + off, ok ? 16 : 0);
                cp16_zfill(dV + r * LD + c, vp + off, ok ? 16 : 0);
            }
            cp_commit();
        };
        __syncthreads();  // the previous query block's tiles are consumed
        if (keyA < keyB) fetch(keyA, 0);
        int buf = 0;
        for (int k0 = keyA; k0 < keyB; k0 += BP, buf ^= 1) {
            const int nkeys = min(BP, keyB - k0);
            const T* sK = sKb + buf * BP * LD;
            const T* sV = sVb + buf * BP * LD;
            if (k0 + BP < keyB) {
                fetch(k0 + BP, buf ^ 1);  // its buffer was released by the barrier that ended tile t - 1
                cp_wait<1>();
            } else {
                cp_wait<0>();
            }
            __syncthreads();  // tile t visible to every warp
            {
                // S[16 x 32] = Q[qb] K[sub..sub+32]^T for this warp's half of the tile
                const int sub = 32 * dh;
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
                // the pair's row maxima over the whole tile
                const int g = lane >> 2;
                float* pm = spm + ((buf * 4 + qb) * 2 + dh) * 16;
                const float* pmo = spm + ((buf * 4 + qb) * 2 + (dh ^ 1)) * 16;
                if ((lane & 3) == 0) {
                    pm[g] = t0;
                    pm[g + 8] = t1;
                }
                pair_sync(qb);
                const float n0m = fmaxf(m0, fmaxf(t0, pmo[g])), n1m = fmaxf(m1, fmaxf(t1, pmo[g + 8]));
                const float c0 = l0 > 0.f ? __expf(m0 - n0m) : 0.f, c1 = l1 > 0.f ? __expf(m1 - n1m) : 0.f;
                m0 = n0m;
                m1 = n1m;
                // P of this half (bf16) into the pair's [16 x 64] tile, its row sums to the pair
                T* P = sP + (buf * 4 + qb) * 16 * PLD;
                float s0 = 0.f, s1 = 0.f;
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
                    const int col = sub + nt * 8 + (lane & 3) * 2;
                    *reinterpret_cast<uint32_t*>(P + g * PLD + col) = pack_bf16(e0[0], e0[1]);
                    *reinterpret_cast<uint32_t*>(P + (g + 8) * PLD + col) = pack_bf16(e1[0], e1[1]);
                }
                s0 += __shfl_xor_sync(0xffffffffu, s0, 1);
                s0 += __shfl_xor_sync(0xffffffffu, s0, 2);
                s1 += __shfl_xor_sync(0xffffffffu, s1, 1);
                s1 += __shfl_xor_sync(0xffffffffu, s1, 2);
                float* ps = sps + ((buf * 4 + qb) * 2 + dh) * 16;
                const float* pso = sps + ((buf * 4 + qb) * 2 + (dh ^ 1)) * 16;
                if ((lane & 3) == 0) {
                    ps[g] = s0;
                    ps[g + 8] = s1;
                }
                pair_sync(qb);
                // both warps of the pair form the same sums (half 0 + half 1)
                const float r0 = dh == 0 ? s0 + pso[g] : pso[g] + s0;
                const float r1 = dh == 0 ? s1 + pso[g + 8] : pso[g + 8] + s1;
                l0 = l0 * c0 + r0;
                l1 = l1 * c1 + r1;
#pragma unroll
                for (int j = 0; j < DH / 8; ++j) {
                    o[j][0] *= c0;
                    o[j][1] *= c0;
                    o[j][2] *= c1;
                    o[j][3] *= c1;
                }
                // O[16 x DH] += P[16 x 64] V[tile][dh*DH ..]
#pragma unroll
                for (int ks = 0; ks < BP / 16; ++ks) {
                    uint32_t a0, a1, a2, a3;
                    ldsm_x4(smem_u32(P + (lane & 15) * PLD + ks * 16 + (lane >> 4) * 8), a0, a1, a2, a3);
#pragma unroll
                    for (int dt = 0; dt < DH / 8; dt += 2) {
                        uint32_t b0, b1, b2, b3;
                        ldsm_x4_t(smem_u32(sV + (ks * 16 + (lane & 7) + ((lane >> 3) & 1) * 8) * LD + dh * DH + dt * 8 +
                                           (lane >> 4) * 8),
                                  b0, b1, b2, b3);
                        mma_bf16(o[dt], a0, a1, a2, a3, b0, b1);
                        mma_bf16(o[dt + 1], a0, a1, a2, a3, b2, b3);
                    }
                }
            }
            __syncthreads();  // every warp is done with buffer `buf` before it is refilled
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
        arrive_rows<D, T>(p, n0, nq, h, 1u);
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
    for (int n0 = 0; n0 < p.N; n0 += NQ) arrive_rows<D, float>(p, n0, min(NQ, p.N - n0), h, KSPLIT);
}

// ------------------------------------------------------------------------- own partials, f32
template <int D>
__device__ void own_block_f32(const RelayParams& p, unsigned char* smem) {
    using T = float;
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
    arrive_rows<D, T>(p, n, 1, h, 1u);
}

// ------------------------------------------------------------------ bf16: own items
// An own CTA (sequence n, head h, 1024-key own block ob) streams its block through a ring of
// OWN_NS stages of OWN_SK keys in shared memory (K rows, then V rows: two bulk copies per stage,
// issued by thread 0, which refills a stage once every warp has released it).  Warp w reads keys
// [w KW, (w + 1) KW) of every stage and runs an online softmax over them; the stage that holds the
// block's end zeroes the keys past it in registers.  The arithmetic runs on packed f32 pairs
// (fma.rn.f32x2: each half is one correctly rounded FMA): products of bf16 values are exact in f32,
// the dot product keeps even and odd elements in two partial sums, and the score is scaled after
// the sum, as the tensor-core prefix path does.  The warps' (max, sum, acc) are merged at the end.
// (A persistent grid streaming several blocks per CTA through the same ring was measured slower:
// the per-key arithmetic bounds the own segment, not the stream.)
constexpr int OWN_SK = 64;    // keys per ring stage
constexpr int OWN_NS = 3;     // ring stages
constexpr int BO_BF16 = 1024; // own keys per bf16 own CTA

template <int D>
struct OwnLayout {
    static constexpr int ROWB = D * 2;                        // bytes of one bf16 key row
    static constexpr int STAGE = 2 * OWN_SK * ROWB;           // K rows, then V rows
    static constexpr int OFF_BAR = OWN_NS * STAGE;            // full[NS], empty[NS]
    static constexpr int OFF_ERR = OFF_BAR + 16 * OWN_NS;
    static constexpr int OFF_ACC = OFF_ERR + 16;              // [NW][D] f32
    static constexpr int BYTES = OFF_ACC + 4 * (THREADS / 32) * D;
};

// Two bf16 (element 2j in the low half) as an f32 pair.
__device__ __forceinline__ float2 bf16x2_f32x2(uint32_t x) {
    return make_float2(__uint_as_float(x << 16), __uint_as_float(x & 0xFFFF0000u));
}
// c = a * b + c on f32 pairs.
__device__ __forceinline__ void ffma2(float2& c, float2 a, float2 b) {
    asm("{.reg .b64 ra, rb, rc;\n\t"
        "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%0, %1};\n\t"
        "fma.rn.f32x2 rc, ra, rb, rc;\n\tmov.b64 {%0, %1}, rc;\n\t}"
        : "+f"(c.x), "+f"(c.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
}
// c = c * s on an f32 pair.
__device__ __forceinline__ void fmul2(float2& c, float s) {
    asm("{.reg .b64 ra, rs;\n\tmov.b64 ra, {%0, %1};\n\tmov.b64 rs, {%2, %2};\n\t"
        "mul.rn.f32x2 ra, ra, rs;\n\tmov.b64 {%0, %1}, ra;\n\t}"
        : "+f"(c.x), "+f"(c.y)
        : "f"(s));
}

template <int D>
__device__ void own_block_bf16(const RelayParams& p, unsigned char* smem) {
    using L = OwnLayout<D>;
    constexpr int EPL = 8;            // bf16 elements per 16-byte lane load
    constexpr int LPK = D / EPL;      // lanes per key row
    constexpr int KPW = 32 / LPK;     // keys per warp instruction
    constexpr int NW = THREADS / 32;
    constexpr int SK = OWN_SK, NS = OWN_NS;
    constexpr int KW = SK / NW;       // keys of one warp in a stage
    constexpr int U = KW / KPW;       // 16-byte loads per lane per stage, K and V each
    constexpr int ROWB = L::ROWB;
    static_assert(KW % KPW == 0 && U >= 1, "stage keys must cover whole warp instructions");
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
    uint64_t* empty = full + NS;
    int* serr = reinterpret_cast<int*>(smem + L::OFF_ERR);
    float* sacc = reinterpret_cast<float*>(smem + L::OFF_ACC);
    __shared__ float s_red[2][NW];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int bid = blockIdx.x - p.H * p.NPB;
    const int ob = bid % p.NOB;
    const int nh = bid / p.NOB;
    const int n = nh / p.H, h = nh - n * p.H;
    const int own = p.own_len ? min(max(p.own_len[n], 0), p.Lo) : p.Lo;
    const int key0 = ob * BO_BF16;
    const int nkeys = max(0, min(BO_BF16, own - key0));
    const size_t row = (size_t)n * p.H + h;
    const int sub = lane / LPK, part = lane % LPK;  // key slot within the warp, chunk of the row
    const __nv_bfloat16* ko = static_cast<const __nv_bfloat16*>(p.ko) + (row * p.Lo + key0) * D;
    const __nv_bfloat16* vo = static_cast<const __nv_bfloat16*>(p.vo) + (row * p.Lo + key0) * D;
    const int nst = (nkeys + SK - 1) / SK;
    if (tid == 0) {
        for (int i = 0; i < NS; ++i) {
            mbar_init(full + i, 1);
            mbar_init(empty + i, NW);
        }
        *serr = 0;
        fence_mbar_init();
    }
    __syncthreads();
    int issued = 0;  // thread 0: stages whose copies were issued
    auto issue = [&](int st) {
        const int k0 = st * SK;
        const uint32_t bytes = (uint32_t)min(SK, nkeys - k0) * ROWB;
        unsigned char* dst = smem + (size_t)(st % NS) * L::STAGE;
        mbar_arrive_expect_tx(full + st % NS, 2 * bytes);
        bulk_g2s(dst, ko + (size_t)k0 * D, bytes, full + st % NS);
        bulk_g2s(dst + SK * ROWB, vo + (size_t)k0 * D, bytes, full + st % NS);
        issued = st + 1;
    };
    if (tid == 0)
        for (int st = 0; st < min(NS, nst); ++st) issue(st);
    float2 q2[EPL / 2];
    {
        const uint4 qx = *reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(p.q) + row * D + part * EPL);
        q2[0] = bf16x2_f32x2(qx.x);
        q2[1] = bf16x2_f32x2(qx.y);
        q2[2] = bf16x2_f32x2(qx.z);
        q2[3] = bf16x2_f32x2(qx.w);
    }
    float m = -FLT_MAX, l = 0.f;
    float2 acc2[EPL / 2];
#pragma unroll
    for (int j = 0; j < EPL / 2; ++j) acc2[j] = make_float2(0.f, 0.f);
    int consumed = 0;
    for (int s = 0; s < nst; ++s) {
        const int slot = s % NS;
        const uint32_t par = (uint32_t)(s / NS) & 1u;
        // warp-uniform: a warp leaves the loop whole if any of its lanes gave up
        if (!__all_sync(0xffffffffu, mbar_wait(full + slot, par, serr, kRelayWaitFull))) break;
        consumed = s + 1;
        const bool tail = (s + 1) * SK > nkeys;  // the stage that holds the block's end (block-uniform)
        const unsigned char* src = smem + (size_t)slot * L::STAGE + (size_t)(warp * KW + sub) * ROWB + part * 16;
        uint4 kr[U], vr[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            kr[u] = *reinterpret_cast<const uint4*>(src + u * KPW * ROWB);
            vr[u] = *reinterpret_cast<const uint4*>(src + SK * ROWB + u * KPW * ROWB);
        }
        if (tail) {  // rows past the block's end hold stale bytes: zero them
#pragma unroll
            for (int u = 0; u < U; ++u)
                if (s * SK + warp * KW + u * KPW + sub >= nkeys) kr[u] = vr[u] = make_uint4(0, 0, 0, 0);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(empty + slot);  // this warp's reads of the slot are done
        if (tid == 0 && s + NS < nst) {
            if (mbar_wait(empty + slot, par, serr, kRelayWaitEmpty)) issue(s + NS);
        }
        float sc[U];
        float mg = -FLT_MAX;
#pragma unroll
        for (int u = 0; u < U; ++u) {
            float2 d2 = make_float2(0.f, 0.f);
            ffma2(d2, q2[0], bf16x2_f32x2(kr[u].x));
            ffma2(d2, q2[1], bf16x2_f32x2(kr[u].y));
            ffma2(d2, q2[2], bf16x2_f32x2(kr[u].z));
            ffma2(d2, q2[3], bf16x2_f32x2(kr[u].w));
            float d = d2.x + d2.y;
#pragma unroll
            for (int o = LPK / 2; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
            sc[u] = d * p.scale;
            if (tail && s * SK + warp * KW + u * KPW + sub >= nkeys) sc[u] = -FLT_MAX;
            mg = fmaxf(mg, sc[u]);
        }
#pragma unroll
        for (int o = LPK; o < 32; o <<= 1) mg = fmaxf(mg, __shfl_xor_sync(0xffffffffu, mg, o));  // every key slot
        const float mn = fmaxf(m, mg);
        const float corr = __expf(m - mn);  // 0 while nothing was seen (acc and l are 0 then)
        l *= corr;
#pragma unroll
        for (int j = 0; j < EPL / 2; ++j) fmul2(acc2[j], corr);
#pragma unroll
        for (int u = 0; u < U; ++u) {
            float w = __expf(sc[u] - mn);
            if (tail && s * SK + warp * KW + u * KPW + sub >= nkeys) w = 0.f;
            if (part == 0) l += w;
            const float2 w2 = make_float2(w, w);
            ffma2(acc2[0], w2, bf16x2_f32x2(vr[u].x));
            ffma2(acc2[1], w2, bf16x2_f32x2(vr[u].y));
            ffma2(acc2[2], w2, bf16x2_f32x2(vr[u].z));
            ffma2(acc2[3], w2, bf16x2_f32x2(vr[u].w));
        }
        m = mn;
    }
    // A block that gave up at a wait still owns the copies it issued: let them land first.
    if (tid == 0) {
        for (int st = consumed; st < issued; ++st) mbar_drain(full + st % NS, (uint32_t)(st / NS) & 1u);
        if (*serr != 0) atomicExch(p.err, *serr);
    }
    float acc[EPL];
#pragma unroll
    for (int j = 0; j < EPL / 2; ++j) {
        acc[2 * j] = acc2[j].x;
        acc[2 * j + 1] = acc2[j].y;
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
    arrive_rows<D, __nv_bfloat16>(p, n, 1, h, 1u);
}

template <int D>
__global__ void __launch_bounds__(THREADS, 2) relay_merge_kernel_bf16(const RelayParams p) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    if ((int)blockIdx.x < p.H * p.NPB) prefix_block_bf16<D>(p, smem_raw, (int)blockIdx.x);
    else own_block_bf16<D>(p, smem_raw);
}


template <int D>
__global__ void __launch_bounds__(THREADS, MIN_BLOCKS_F32) relay_merge_kernel_f32(const RelayParams p) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    if ((int)blockIdx.x < p.H * p.NPB) prefix_block_f32<D>(p, smem_raw);
    else own_block_f32<D>(p, smem_raw);
}

size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

struct Layout {
    int NPB, NOB, P, bpc, ppc, bo;
    size_t off_acc, off_max, off_sum, off_cnt, n_cnt, total;
};

// bf16: one partial per 1024-key prefix CTA and per 1024-key own CTA; f32: two partials per 64-key
// prefix CTA and one per 1024-key own CTA; one arrival counter per (n, h) row.
Layout layout(int64_t N, int64_t H, int64_t D, int64_t Lp, int64_t Lo, bool bf16) {
    Layout L{};
    L.bpc = bf16 ? BP * TILES_BF16 : BP;
    L.ppc = bf16 ? 1 : KSPLIT;
    L.bo = bf16 ? BO_BF16 : BO;
    L.NPB = (int)((Lp + L.bpc - 1) / L.bpc);
    L.NOB = (int)((Lo + L.bo - 1) / L.bo);
    if (L.NOB == 0) L.NOB = 1;  // one (empty) own partial keeps the arrival count uniform
    L.P = L.NPB * L.ppc + L.NOB;
    const size_t rows = (size_t)N * H;
    L.off_acc = 0;
    L.off_max = align_up(L.off_acc + rows * L.P * D * sizeof(float), 256);
    L.off_sum = align_up(L.off_max + rows * L.P * sizeof(float), 256);
    L.off_cnt = align_up(L.off_sum + rows * L.P * sizeof(float), 256);
    L.n_cnt = rows;
    L.total = align_up(L.off_cnt + L.n_cnt * sizeof(unsigned), 256);
    return L;
}

template <int D>
size_t relay_smem_f32() {
    const size_t prefix = sizeof(float) * (size_t)((BP / KSPLIT) * (D + 1) + (BP / KSPLIT) * D + 32 * (D + 1) + 32 * (BP / KSPLIT + 1));
    const size_t own = sizeof(float) * (size_t)(BO + (THREADS / 32) * D);
    return prefix > own ? prefix : own;
}
template <int D>
size_t relay_smem_bf16() {
    const size_t prefix = sizeof(__nv_bfloat16) * ((size_t)(NQ + 4 * BP) * (D + PAD) + 2 * 4 * 16 * PLD) +
                          sizeof(float) * 2 * (2 * 4 * 2 * 16);
    const size_t own = OwnLayout<D>::BYTES;
    return prefix > own ? prefix : own;
}

template <int D>
int launch_relay_f32(const RelayParams& p, cudaStream_t st) {
    const size_t smem = relay_smem_f32<D>();
    cudaError_t e = cudaFuncSetAttribute(relay_merge_kernel_f32<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return cuda_status(e, "relay: cudaFuncSetAttribute");
    const unsigned grid = (unsigned)(p.H * p.NPB + p.N * p.H * p.NOB);
    relay_merge_kernel_f32<D><<<grid, THREADS, smem, st>>>(p);
    return launch_status("relay_merge_kernel_f32");
}

template <int D>
int launch_relay_bf16(const RelayParams& p, cudaStream_t st) {
    const size_t smem = relay_smem_bf16<D>();
    cudaError_t e = cudaFuncSetAttribute(relay_merge_kernel_bf16<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return cuda_status(e, "relay: cudaFuncSetAttribute");
    const unsigned grid = (unsigned)(p.H * p.NPB + p.N * p.H * p.NOB);
    relay_merge_kernel_bf16<D><<<grid, THREADS, smem, st>>>(p);
    return launch_status("relay_merge_kernel_bf16");
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
    p.bo = L.bo;
    int rc = device_error_record(&p.err);
    if (rc != DBL_OK) return rc;
    cudaError_t e = cudaMemsetAsync(p.counter, 0, sizeof(unsigned) * L.n_cnt, st);
    if (e != cudaSuccess) return cuda_status(e, "relay: clear counters");
    const bool bf = a->dtype == DBL_BF16;
    if (a->head_dim == 128) return bf ? launch_relay_bf16<128>(p, st) : launch_relay_f32<128>(p, st);
    return bf ? launch_relay_bf16<64>(p, st) : launch_relay_f32<64>(p, st);
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
