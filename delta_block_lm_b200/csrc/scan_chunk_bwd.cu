// Chunked backward of the stateful GDN-2 scan (gdn_training_backward, gdn_training.rs:117-284) for
// 16-token checkpoints, the reverse of the chunked forward in scan_chunk.cu.
//
// Per chunk the forward is E = U0 - B' S0, O = Q' S0 + M E, S_end = diag(P_last) S0 + Wd^T E and
// scores |k_t| |E_t| (maps as in scan_chunk.cu).  Its vector-Jacobian product:
//   dE    = M^T dO + g E + Wd dS_end             (g_t = g_score_t |k_t| / |E_t| where both norms > 0)
//   dS0   = G^T dS_end + Hb,   Hb = Q'^T dO - B'^T (M^T dO + g E),   G = diag(P_last) - Wd^T B'
//   dWV   = Ti^T dE,  dQ' = dO S0^T,  dB = -dWV S0^T,  dM = lower(dO E^T),  dA = -strict_lower(dWV E^T),
//   dWd   = E dS_end^T,  dP_last = rowsum(S0 (.) dS_end)
// (dA and dB follow from E = Ti (WV - B S0) without differentiating the inverse), and through the
// chunk's products d[t][s] = f_{s+1} ... f_t, per key channel i:
//   dq_t  = dQ'_t P_t + sum_{s<=t} dM[t][s] d[t][s] k_s
//   d(ek)_t = dB_t P_t + sum_{s<t} dA[t][s] d[t][s] k_s
//   dk_s  = sum_{t>s} (dA[t][s] ek_t + dM[t][s] q_t) d[t][s] + dM[s][s] q_s + dWd_s d[last][s]
//   dP_t  = dQ'_t q_t + dB_t ek_t (+ dP_last for the last token)
//   df_u  = sum_{t>=u} d[t][u] Y[t][u],  Y[t][u] = dP_t P_{u-1} + sum_{s<u} DD[t][s] d[u-1][s],
//           DD[t][s] = (dA[t][s] ek_t + dM[t][s] q_t + [t last] dWd_s) k_s
// with every product formed directly (no division by a decay, so resets and zero gates are exact),
// then d alpha = df (valid, not reset), d erase = d(ek) k, dk += d(ek) erase + g_score |E| k / |k|,
// dv = dWV write, d write = dWV v.
//
// Kernels: the chunked forward (maps kept, chunk-start states, edits), chunk_bwd_pre_kernel (per
// chunk: dE_pre = M^T dO + g E, Hb, G^T), chunk_bwd_rev_kernel (per (b, h, column group), chunks
// from the last: dE and dS_end, the adjoint state in shared memory), chunk_bwd_grad_kernel (per
// chunk: every input gradient).
#include "scan_chunk.cuh"
#include "scan_seq_params.cuh"

#include <atomic>

namespace dbl {
namespace {

using namespace chunk;

struct CBwdParams {
    int B, T, H, K, V, nch;
    const float *q, *k, *v, *alpha, *erase, *write, *valid, *reset;
    const float *g_out, *g_fin, *g_score;
    float *dq, *dk, *dv, *dalpha, *derase, *dwrite, *dinitial;
    const float* fwd;    // forward chunk maps (with the backward's extra maps)
    const float* ck;     // chunk-start states [B*H][nch][K][V]
    const float* edits;  // [B,T,H,V]
    float* rev;          // reverse-pass maps per chunk
    float* dE;           // [B*H][nch][16][V]
    float* dSe;          // adjoint of each chunk's end state [B*H][nch][K][V]
};

// Reverse-pass maps of one chunk: the part every column group reads (Wd, G^T with rows of KP, zero
// beyond K; |E_t|) then the column-sliced part (dE_pre, Hb as rows of V).
struct RevBlock {
    int kp, wd, gt, en, sh, dep, hb, total;
};
__host__ __device__ inline RevBlock rev_block(int K, int V) {
    RevBlock L{};
    L.kp = ((K + 3) & ~3) + 4;
    int o = 0;
    L.wd = o; o += CC * L.kp;
    L.gt = o; o += K * L.kp;
    L.en = o; o += CC;
    L.sh = o;
    L.dep = o; o += CC * V;
    L.hb = o; o += K * V;
    L.total = (o + 3) & ~3;
    return L;
}

// acc[r][c] += sum_{s < kd} A[(r0 + r) lda + s] Bm[s ldb + n0 + c] for a 2 x 4 tile (tile_mm with a
// contraction length kd, a multiple of 4)
__device__ __forceinline__ void tile_mmk(float (&acc)[2][4], const float* A, int lda, int r0, const float* Bm,
                                         int ldb, int n0, int kd) {
#pragma unroll 2
    for (int s = 0; s < kd; s += 4) {
        const float4 b0 = lds4(Bm + (s + 0) * ldb + n0), b1 = lds4(Bm + (s + 1) * ldb + n0);
        const float4 b2 = lds4(Bm + (s + 2) * ldb + n0), b3 = lds4(Bm + (s + 3) * ldb + n0);
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const float4 a = lds4(A + (r0 + r) * lda + s);
            acc[r][0] = fmaf(a.x, b0.x, fmaf(a.y, b1.x, fmaf(a.z, b2.x, fmaf(a.w, b3.x, acc[r][0]))));
            acc[r][1] = fmaf(a.x, b0.y, fmaf(a.y, b1.y, fmaf(a.z, b2.y, fmaf(a.w, b3.y, acc[r][1]))));
            acc[r][2] = fmaf(a.x, b0.z, fmaf(a.y, b1.z, fmaf(a.z, b2.z, fmaf(a.w, b3.z, acc[r][2]))));
            acc[r][3] = fmaf(a.x, b0.w, fmaf(a.y, b1.w, fmaf(a.z, b2.w, fmaf(a.w, b3.w, acc[r][3]))));
        }
    }
}

__device__ __forceinline__ size_t tok(const CBwdParams& p, int b, int t, int h) {
    return ((size_t)b * p.T + t) * p.H + h;
}

// ------------------------------------------------------------------------------------------------
// Per chunk: |E_t|, g_t, dE_pre = M^T dO + g E, Hb = Q'^T dO - B'^T dE_pre, Wd and G^T.
template <int KMAX>
__global__ void __launch_bounds__(CTH) chunk_bwd_pre_kernel(const CBwdParams p) {
    constexpr int SR = CC + 4;
    __shared__ __align__(16) float sMT[CC][SR], sQpT[KMAX][SR], sBpT[KMAX][SR];
    __shared__ __align__(16) float sdO[CC][CVMAX], sE[CC][CVMAX], sdep[CC][CVMAX];
    __shared__ float sgE[CC], sen[CC];
    __shared__ int sact[CC];
    const int K = p.K, V = p.V, K4 = (K + 3) & ~3, V4 = (V + 3) & ~3;
    const int nch = p.nch;
    const int c = blockIdx.x % nch, bh = blockIdx.x / nch, b = bh / p.H, h = bh - (bh / p.H) * p.H;
    const int t0 = c * CC, n = min(CC, p.T - t0);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const ChunkBlock F = chunk_block(K, V, true);
    const RevBlock R = rev_block(K, V);
    const float* fb = p.fwd + ((size_t)bh * nch + c) * F.total;
    float* rb = p.rev + ((size_t)bh * nch + c) * R.total;
    const int KP = F.kp;

    // every global load of the kernel is issued before the first barrier: the token flags, score
    // gradients and |k_t|, the maps (M, Q', B' transposed), dO and the edits; the Wd and G^T rows of
    // the reverse block are plain copies
    __shared__ float sgs[CC], skn[CC];
    if (tid < CC) {
        const bool act = tid < n && p.valid[(size_t)b * p.T + t0 + tid] != 0.f;
        sact[tid] = act;
        sgs[tid] = (p.g_score && act) ? p.g_score[tok(p, b, t0 + tid, h)] : 0.f;
        skn[tid] = fb[F.kn + tid];
    }
    for (int x = tid; x < CC * CC; x += CTH) {
        const int t = x / CC, s = x - t * CC;
        sMT[s][t] = fb[F.mm + x];
    }
    // Q' and B' rows (KP floats, zero beyond K, 16-byte aligned) four floats at a time, stored transposed
    for (int x = tid; x < CC * (KMAX / 4); x += CTH) {
        const int t = x / (KMAX / 4), i = 4 * (x - t * (KMAX / 4));
        const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
        const float4 qv = i < KP ? *reinterpret_cast<const float4*>(fb + F.qp + t * KP + i) : z4;
        const float4 bv = i < KP ? *reinterpret_cast<const float4*>(fb + F.bp + t * KP + i) : z4;
        sQpT[i][t] = qv.x;
        sQpT[i + 1][t] = qv.y;
        sQpT[i + 2][t] = qv.z;
        sQpT[i + 3][t] = qv.w;
        sBpT[i][t] = bv.x;
        sBpT[i + 1][t] = bv.y;
        sBpT[i + 2][t] = bv.z;
        sBpT[i + 3][t] = bv.w;
    }
    if ((V & 3) == 0 && (reinterpret_cast<uintptr_t>(p.g_out) & 15) == 0) {
        for (int x = tid; x < CC * (CVMAX / 4); x += CTH) {
            const int t = x / (CVMAX / 4), j = 4 * (x - t * (CVMAX / 4));
            const bool in = t < n && j < V;
            const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
            float4 dov = z4, ev = z4;
            if (in) {
                ev = *reinterpret_cast<const float4*>(p.edits + tok(p, b, t0 + t, h) * V + j);
                if (p.valid[(size_t)b * p.T + t0 + t] != 0.f)
                    dov = *reinterpret_cast<const float4*>(p.g_out + tok(p, b, t0 + t, h) * V + j);
            }
            *reinterpret_cast<float4*>(&sdO[t][j]) = dov;
            *reinterpret_cast<float4*>(&sE[t][j]) = ev;
        }
    } else {
        for (int x = tid; x < CC * CVMAX; x += CTH) {
            const int t = x / CVMAX, j = x - t * CVMAX;
            const bool in = t < n && j < V;
            const bool act = in && p.valid[(size_t)b * p.T + t0 + t] != 0.f;
            sdO[t][j] = act ? p.g_out[tok(p, b, t0 + t, h) * V + j] : 0.f;
            sE[t][j] = in ? p.edits[tok(p, b, t0 + t, h) * V + j] : 0.f;
        }
    }
    for (int x = tid; x < CC * KP / 4; x += CTH)
        reinterpret_cast<float4*>(rb + R.wd)[x] = reinterpret_cast<const float4*>(fb + F.wd)[x];
    for (int x = tid; x < K * KP; x += CTH) {
        const int i = x / KP, i2 = x - i * KP;
        rb[R.gt + x] = i2 < K ? fb[F.g + i2 * KP + i] : 0.f;
    }
    __syncthreads();
    for (int t = warp; t < CC; t += CTH / 32) {
        float e2 = 0.f;
        for (int j = lane; j < V; j += 32) e2 = fmaf(sE[t][j], sE[t][j], e2);
        e2 = warp_sum(e2);
        if (lane == 0) {
            const float en = sqrtf(e2), kn = skn[t];
            sen[t] = en;
            sgE[t] = (sact[t] && en > 0.f && kn > 0.f) ? sgs[t] * kn / en : 0.f;
        }
    }
    __syncthreads();
    // dE_pre (2 x 4 tiles)
    const int nv = V4 / 4;
    for (int x = tid; x < (CC / 2) * nv; x += CTH) {
        const int r0 = 2 * (x / nv), n0 = 4 * (x - (x / nv) * nv);
        float acc[2][4] = {};
        tile_mm(acc, &sMT[0][0], SR, r0, &sdO[0][0], CVMAX, n0);
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            float d[4];
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) {
                d[cc] = fmaf(sgE[r0 + r], sE[r0 + r][n0 + cc], acc[r][cc]);
                sdep[r0 + r][n0 + cc] = d[cc];
            }
            float* dst = rb + R.dep + (r0 + r) * V + n0;
            if ((V & 3) == 0) {
                *reinterpret_cast<float4*>(dst) = make_float4(d[0], d[1], d[2], d[3]);
            } else {
#pragma unroll
                for (int cc = 0; cc < 4; ++cc)
                    if (n0 + cc < V) dst[cc] = d[cc];
            }
        }
    }
    __syncthreads();
    // Hb = Q'^T dO - B'^T dE_pre, rows i < K
    const int rk = (K + 1) / 2;
    for (int x = tid; x < rk * nv; x += CTH) {
        const int r0 = 2 * (x / nv), n0 = 4 * (x - (x / nv) * nv);
        float a1[2][4] = {}, a2[2][4] = {};
        tile_mm(a1, &sQpT[0][0], SR, r0, &sdO[0][0], CVMAX, n0);
        tile_mm(a2, &sBpT[0][0], SR, r0, &sdep[0][0], CVMAX, n0);
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            if (r0 + r >= K) continue;
            float* dst = rb + R.hb + (r0 + r) * V + n0;
            if ((V & 3) == 0) {
                *reinterpret_cast<float4*>(dst) = make_float4(a1[r][0] - a2[r][0], a1[r][1] - a2[r][1],
                                                              a1[r][2] - a2[r][2], a1[r][3] - a2[r][3]);
            } else {
#pragma unroll
                for (int cc = 0; cc < 4; ++cc)
                    if (n0 + cc < V) dst[cc] = a1[r][cc] - a2[r][cc];
            }
        }
    }
    // |E_t|
    if (tid < CC) rb[R.en + tid] = sen[tid];
    (void)K4;
}

// ------------------------------------------------------------------------------------------------
// The reverse pass: one CTA per (b, h, column group), chunks from the last, the adjoint state dS
// [K4][VG] in shared memory (double-buffered), the reverse maps in a cp.async ring.  At chunk c,
// dS is the adjoint of the chunk's end state: it is written out, dE = dE_pre + Wd dS, and dS
// becomes G^T dS + Hb.
template <int KMAX, int VG>
__global__ void __launch_bounds__(CTH) chunk_bwd_rev_kernel(const CBwdParams p, int ngroups, int NB) {
    constexpr int RP = CTH / VG;
    constexpr int NT = CC / RP;
    constexpr int NS = KMAX / RP;
    extern __shared__ __align__(16) float smem_rev[];
    const int K = p.K, V = p.V, K4 = (K + 3) & ~3;
    const int nch = p.nch;
    const int grp = blockIdx.x % ngroups, bh = blockIdx.x / ngroups;
    const int b = bh / p.H, h = bh - (bh / p.H) * p.H;
    const int c0 = grp * VG, vg = min(VG, V - c0);
    const int tid = threadIdx.x, j = tid % VG, rr = tid / VG;
    const RevBlock L = rev_block(K, V);
    const int KP = L.kp;
    const int rows = CC + K;  // dE_pre, Hb rows
    const int bfl = L.sh + rows * VG;
    float* Sb0 = smem_rev;
    float* Sb1 = smem_rev + K4 * VG;
    float* bb0 = smem_rev + 2 * K4 * VG;
    const bool vec = (V & 3) == 0;
    const size_t sbase = ((size_t)b * p.H + h) * K * V;
    for (int x = tid; x < K4 * VG; x += CTH) {
        const int i = x / VG, jj = x - i * VG;
        Sb0[x] = (p.g_fin && i < K && jj < vg) ? p.g_fin[sbase + (size_t)i * V + c0 + jj] : 0.f;
        Sb1[x] = 0.f;
    }
    // this thread's copies of the column-sliced part (dE_pre, Hb rows), the same every chunk:
    // shared-memory and block offsets (16-byte copies when V is a multiple of 4); a thread's copies
    // are a prefix of its slots
    constexpr int MAXCOL = ((CC + KMAX) * VG + CTH - 1) / CTH;  // rows x columns over the threads
    int soff[MAXCOL], goff[MAXCOL];
    const int per = vec ? vg >> 2 : vg, ncopy = rows * per;
#pragma unroll
    for (int k = 0; k < MAXCOL; ++k) {
        const int x = tid + k * CTH;
        const int r = x / per, w = x - r * per;
        soff[k] = L.sh + r * VG + (vec ? 4 * w : w);
        goff[k] = L.sh + r * V + c0 + (vec ? 4 * w : w);
    }
    // stages the maps of reverse step `it` (chunk nch - 1 - it) into buffer it % NB, one group each
    auto prefetch = [&](int it) {
        if (it < nch) {
            const int c = nch - 1 - it;
            const float* src = p.rev + ((size_t)bh * nch + c) * L.total;
            float* dst = bb0 + (it % NB) * bfl;
            for (int x = tid; x < L.sh / 4; x += CTH) cp_async16(dst + 4 * x, src + 4 * x);
#pragma unroll
            for (int k = 0; k < MAXCOL; ++k) {
                if (tid + k * CTH >= ncopy) break;
                if (vec) cp_async16(dst + soff[k], src + goff[k]);
                else cp_async4(dst + soff[k], src + goff[k]);
            }
        }
        cp_async_commit();
    };
    for (int it = 0; it < NB - 1; ++it) prefetch(it);
    for (int it = 0; it < nch; ++it) {
        const int c = nch - 1 - it;
        const int n = min(CC, p.T - c * CC);
        cp_async_wait_pending(NB - 2);
        __syncthreads();
        prefetch(it + NB - 1);
        const float* blk = bb0 + (it % NB) * bfl;
        const float* S = (it & 1) ? Sb1 : Sb0;
        float* Sn = (it & 1) ? Sb0 : Sb1;
        const float* wd = blk + L.wd;
        const float* gt = blk + L.gt;
        const float* dep = blk + L.sh;
        const float* hb = dep + CC * VG;
        // the adjoint of this chunk's end state
        if (j < vg) {
            float* ds = p.dSe + ((size_t)bh * nch + c) * K * V + c0 + j;
#pragma unroll
            for (int m = 0; m < NS; ++m)
                if (rr + m * RP < K) ds[(size_t)(rr + m * RP) * V] = S[(rr + m * RP) * VG + j];
        }
        float o[NT], acc[NS];
#pragma unroll
        for (int m = 0; m < NT; ++m) o[m] = dep[(rr + m * RP) * VG + j];
#pragma unroll
        for (int m = 0; m < NS; ++m) acc[m] = (rr + m * RP < K) ? hb[(rr + m * RP) * VG + j] : 0.f;
        // unrolled over the compile-time key bound (K4 <= KMAX) so that the loads issue early
#pragma unroll
        for (int i = 0; i < KMAX; i += 4) {
            if (i >= K4) break;
            const float s0 = S[(i + 0) * VG + j], s1 = S[(i + 1) * VG + j];
            const float s2 = S[(i + 2) * VG + j], s3 = S[(i + 3) * VG + j];
#pragma unroll
            for (int m = 0; m < NT; ++m) {
                const float4 wv = lds4(wd + (rr + m * RP) * KP + i);
                o[m] = fmaf(wv.x, s0, fmaf(wv.y, s1, fmaf(wv.z, s2, fmaf(wv.w, s3, o[m]))));
            }
#pragma unroll
            for (int m = 0; m < NS; ++m) {
                if (rr + m * RP < K) {
                    const float4 gv = lds4(gt + (rr + m * RP) * KP + i);
                    acc[m] = fmaf(gv.x, s0, fmaf(gv.y, s1, fmaf(gv.z, s2, fmaf(gv.w, s3, acc[m]))));
                }
            }
        }
#pragma unroll
        for (int m = 0; m < NS; ++m)
            if (rr + m * RP < K) Sn[(rr + m * RP) * VG + j] = acc[m];
#pragma unroll
        for (int m = 0; m < NT; ++m) {
            const int t = rr + m * RP;
            if (t < n && j < vg) p.dE[(((size_t)bh * nch + c) * CC + t) * V + c0 + j] = o[m];
        }
    }
    __syncthreads();
    if (p.dinitial) {
        const float* S = (nch & 1) ? Sb1 : Sb0;
        for (int x = tid; x < K * vg; x += CTH) {
            const int i = x / vg, jj = x - i * vg;
            p.dinitial[sbase + (size_t)i * V + c0 + jj] = S[i * VG + jj];
        }
    }
}

// ------------------------------------------------------------------------------------------------
// Per chunk: every input gradient (see the top of the file).  Shared memory carve-up, in floats;
// rows of value width use the stride CV = V4 + 4.
// S0, dS_end and E are also kept transposed (contraction index as the row: S0T [V4][KT],
// dST [V4][KT], ET [V4][CC + 4]) so that every product is a tile_mm whose consecutive lanes read
// consecutive float4s of the B operand.
struct GradSmem {
    int cv, kt, k, q, ek, f, er, P, tit, E, dE, dO, dWV, S0T, dST, ET, dQp, dB, dWd, dP, dM, dA, dPl, en, kn, gs,
        act, rst, C, total;
};
__host__ __device__ inline GradSmem grad_smem(int kmax, int V) {
    GradSmem L{};
    const int V4 = (V + 3) & ~3;
    L.cv = V4 + 4;
    L.kt = kmax + 4;
    const int tk = CC * kmax, tv = CC * L.cv, sr = CC * (CC + 4);
    int o = 0;
    L.k = o; o += tk;
    L.q = o; o += tk;
    L.ek = o; o += tk;
    L.f = o; o += tk;
    L.er = o; o += tk;
    L.P = o; o += tk;
    L.tit = o; o += sr;
    L.E = o; o += tv;
    L.dE = o; o += tv;
    L.dO = o; o += tv;
    L.dWV = o; o += tv;
    L.S0T = o; o += V4 * L.kt;
    L.dST = o; o += V4 * L.kt;
    L.ET = o; o += V4 * (CC + 4);
    L.dQp = o; o += tk;
    L.dB = o; o += tk;
    L.dWd = o; o += tk;
    L.dP = o; o += tk;
    L.dM = o; o += sr;
    L.dA = o; o += sr;
    L.dPl = o; o += kmax;
    L.en = o; o += CC;
    L.kn = o; o += CC;
    L.gs = o; o += CC;
    L.act = o; o += CC;
    L.rst = o; o += CC;
    // phase 4's terms C [CC][CC][kmax] reuse E .. dS_end when those are large enough
    if (L.ET - L.E >= CC * CC * kmax) {
        L.C = L.E;
    } else {
        o = (o + 3) & ~3;
        L.C = o; o += CC * CC * kmax;
    }
    L.total = o;
    return L;
}

// 512 threads: each phase's work items (up to 320 tiles, 16 x K channel walks) fit in one round
constexpr int GTH = 512;

template <int KMAX>
__global__ void __launch_bounds__(GTH, 2) chunk_bwd_grad_kernel(const CBwdParams p) {
    constexpr int SR = CC + 4;
    extern __shared__ __align__(16) float smem_g[];
    const int K = p.K, V = p.V, K4 = (K + 3) & ~3, V4 = (V + 3) & ~3;
    const int nch = p.nch;
    const int c = blockIdx.x % nch, bh = blockIdx.x / nch, b = bh / p.H, h = bh - (bh / p.H) * p.H;
    const int t0 = c * CC, n = min(CC, p.T - t0);
    const int tid = threadIdx.x;
    const GradSmem L = grad_smem(KMAX, V);
    const int CV = L.cv;
    float(*sk)[KMAX] = reinterpret_cast<float(*)[KMAX]>(smem_g + L.k);
    float(*sq)[KMAX] = reinterpret_cast<float(*)[KMAX]>(smem_g + L.q);
    float(*sek)[KMAX] = reinterpret_cast<float(*)[KMAX]>(smem_g + L.ek);
    float(*sf)[KMAX] = reinterpret_cast<float(*)[KMAX]>(smem_g + L.f);
    float(*ser)[KMAX] = reinterpret_cast<float(*)[KMAX]>(smem_g + L.er);
    float(*sP)[KMAX] = reinterpret_cast<float(*)[KMAX]>(smem_g + L.P);
    float(*sdQp)[KMAX] = reinterpret_cast<float(*)[KMAX]>(smem_g + L.dQp);
    float(*sdB)[KMAX] = reinterpret_cast<float(*)[KMAX]>(smem_g + L.dB);
    float(*sdWd)[KMAX] = reinterpret_cast<float(*)[KMAX]>(smem_g + L.dWd);
    float(*sdP)[KMAX] = reinterpret_cast<float(*)[KMAX]>(smem_g + L.dP);
    float(*sdM)[SR] = reinterpret_cast<float(*)[SR]>(smem_g + L.dM);
    float(*sdA)[SR] = reinterpret_cast<float(*)[SR]>(smem_g + L.dA);
    float* sTiT = smem_g + L.tit;
    float* sE = smem_g + L.E;
    float* sdE = smem_g + L.dE;
    float* sdO = smem_g + L.dO;
    float* sdWV = smem_g + L.dWV;
    float* sS0T = smem_g + L.S0T;
    float* sdST = smem_g + L.dST;
    float* sET = smem_g + L.ET;
    const int KT = L.kt;
    float* sdPl = smem_g + L.dPl;
    float* sen = smem_g + L.en;
    float* skn = smem_g + L.kn;
    float* sgs = smem_g + L.gs;
    int* sact = reinterpret_cast<int*>(smem_g + L.act);
    int* srst = reinterpret_cast<int*>(smem_g + L.rst);
    const ChunkBlock F = chunk_block(K, V, true);
    const RevBlock R = rev_block(K, V);
    const float* fb = p.fwd + ((size_t)bh * nch + c) * F.total;
    const float* rb = p.rev + ((size_t)bh * nch + c) * R.total;
    const int KP = F.kp;

    if (tid < CC) {
        const bool in = tid < n;
        const int t = t0 + tid;
        sact[tid] = in && p.valid[(size_t)b * p.T + t] != 0.f;
        srst[tid] = in && p.reset[(size_t)b * p.T + t] != 0.f;
        sen[tid] = rb[R.en + tid];
        skn[tid] = fb[F.kn + tid];
        sgs[tid] = (in && p.g_score) ? p.g_score[tok(p, b, t, h)] : 0.f;
    }
    for (int x = tid; x < CC * SR; x += GTH) {
        const int t = x / SR, s = x - t * SR;
        sTiT[x] = s < CC ? fb[F.ti + s * CC + t] : 0.f;
    }
    // no barrier yet: the token flags are read again where needed, so every load is in flight at once.
    // Rows are read four floats at a time where widths and pointers allow (K, V multiples of 4).
    auto a16 = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0; };
    const bool vk = (K & 3) == 0 && a16(p.k) && a16(p.q) && a16(p.erase) && a16(p.alpha);
    const bool vv = (V & 3) == 0 && a16(p.g_out);
    if (vk) {
        for (int x = tid; x < CC * (KMAX / 4); x += GTH) {
            const int u = x / (KMAX / 4), i = 4 * (x - u * (KMAX / 4));
            const int t = t0 + u;
            const bool act = u < n && p.valid[(size_t)b * p.T + t] != 0.f;
            const bool rst = u < n && p.reset[(size_t)b * p.T + t] != 0.f;
            const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
            float4 kv = z4, qv = z4, f = make_float4(1.f, 1.f, 1.f, 1.f), e = z4, pv = z4;
            if (u < n && i < K) {
                const size_t gi = tok(p, b, t, h) * K + i;
                kv = *reinterpret_cast<const float4*>(p.k + gi);
                if (act) {
                    qv = *reinterpret_cast<const float4*>(p.q + gi);
                    e = *reinterpret_cast<const float4*>(p.erase + gi);
                    f = rst ? z4 : *reinterpret_cast<const float4*>(p.alpha + gi);
                }
            }
            if (i < K) pv = *reinterpret_cast<const float4*>(fb + F.pp + u * KP + i);
            *reinterpret_cast<float4*>(&sk[u][i]) = kv;
            *reinterpret_cast<float4*>(&sq[u][i]) = qv;
            *reinterpret_cast<float4*>(&sf[u][i]) = f;
            *reinterpret_cast<float4*>(&ser[u][i]) = e;
            *reinterpret_cast<float4*>(&sek[u][i]) = make_float4(e.x * kv.x, e.y * kv.y, e.z * kv.z, e.w * kv.w);
            *reinterpret_cast<float4*>(&sP[u][i]) = pv;
        }
    }
    for (int x = tid; x < (vk ? 0 : CC * KMAX); x += GTH) {
        const int u = x / KMAX, i = x - u * KMAX;
        const int t = t0 + u;
        const bool act = u < n && p.valid[(size_t)b * p.T + t] != 0.f;
        const bool rst = u < n && p.reset[(size_t)b * p.T + t] != 0.f;
        float kv = 0.f, qv = 0.f, f = 1.f, e = 0.f, pv = 0.f;
        if (u < n && i < K) {
            const size_t gi = tok(p, b, t, h) * K + i;
            kv = p.k[gi];
            if (act) {
                qv = p.q[gi];
                e = p.erase[gi];
                f = rst ? 0.f : p.alpha[gi];
            }
        }
        if (i < K) pv = fb[F.pp + u * KP + i];
        sk[u][i] = kv;
        sq[u][i] = qv;
        sf[u][i] = f;
        ser[u][i] = e;
        sek[u][i] = e * kv;
        sP[u][i] = pv;
    }
    if (vv) {
        for (int x = tid; x < CC * (CV / 4); x += GTH) {
            const int t = x / (CV / 4), j = 4 * (x - t * (CV / 4));
            const bool in = t < n && j < V;
            const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
            float4 ev = z4, de = z4, dov = z4;
            if (in) {
                ev = *reinterpret_cast<const float4*>(p.edits + tok(p, b, t0 + t, h) * V + j);
                de = *reinterpret_cast<const float4*>(p.dE + (((size_t)bh * nch + c) * CC + t) * V + j);
                if (p.valid[(size_t)b * p.T + t0 + t] != 0.f)
                    dov = *reinterpret_cast<const float4*>(p.g_out + tok(p, b, t0 + t, h) * V + j);
            }
            *reinterpret_cast<float4*>(sE + t * CV + j) = ev;
            *reinterpret_cast<float4*>(sdE + t * CV + j) = de;
            *reinterpret_cast<float4*>(sdO + t * CV + j) = dov;
            if (j < V4) {
                sET[(j + 0) * SR + t] = ev.x;
                sET[(j + 1) * SR + t] = ev.y;
                sET[(j + 2) * SR + t] = ev.z;
                sET[(j + 3) * SR + t] = ev.w;
            }
        }
        // transposed: consecutive threads read consecutive columns of one state row
        for (int x = tid; x < KT * (V4 / 4); x += GTH) {
            const int i = x / (V4 / 4), j = 4 * (x - i * (V4 / 4));
            const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
            float4 a = z4, g = z4;
            if (i < K) {
                const size_t gi = ((size_t)bh * nch + c) * K * V + (size_t)i * V + j;
                a = *reinterpret_cast<const float4*>(p.ck + gi);
                g = *reinterpret_cast<const float4*>(p.dSe + gi);
            }
            sS0T[(j + 0) * KT + i] = a.x;
            sS0T[(j + 1) * KT + i] = a.y;
            sS0T[(j + 2) * KT + i] = a.z;
            sS0T[(j + 3) * KT + i] = a.w;
            sdST[(j + 0) * KT + i] = g.x;
            sdST[(j + 1) * KT + i] = g.y;
            sdST[(j + 2) * KT + i] = g.z;
            sdST[(j + 3) * KT + i] = g.w;
        }
    }
    for (int x = tid; x < (vv ? 0 : CC * CV); x += GTH) {
        const int t = x / CV, j = x - t * CV;
        const bool in = t < n && j < V;
        const float ev = in ? p.edits[tok(p, b, t0 + t, h) * V + j] : 0.f;
        sE[x] = ev;
        if (j < V4) sET[j * SR + t] = ev;
        sdE[x] = in ? p.dE[(((size_t)bh * nch + c) * CC + t) * V + j] : 0.f;
        sdO[x] = (in && p.valid[(size_t)b * p.T + t0 + t] != 0.f) ? p.g_out[tok(p, b, t0 + t, h) * V + j] : 0.f;
    }
    // transposed: consecutive threads read consecutive j of one state row
    for (int x = tid; x < (vv ? 0 : KT * V4); x += GTH) {
        const int i = x / V4, j = x - i * V4;
        const bool in = i < K && j < V;
        sS0T[j * KT + i] = in ? p.ck[((size_t)bh * nch + c) * K * V + (size_t)i * V + j] : 0.f;
        sdST[j * KT + i] = in ? p.dSe[((size_t)bh * nch + c) * K * V + (size_t)i * V + j] : 0.f;
    }
    __syncthreads();
    // phase 1: dWV = Ti^T dE, dQ' = dO S0^T, dM = lower(dO E^T), dWd = E dS^T, dP_last
    {
        const int nv = V4 / 4, nk = K4 / 4;
        const int t1 = (CC / 2) * nv, t2 = (CC / 2) * nk, t3 = (CC / 2) * (CC / 4), t4 = (CC / 2) * nk;
        for (int x = tid; x < t1 + t2 + t3 + t4 + K; x += GTH) {
            float acc[2][4] = {};
            int y = x;
            if (y < t1) {
                const int r0 = 2 * (y / nv), n0 = 4 * (y - (y / nv) * nv);
                tile_mm(acc, sTiT, SR, r0, sdE, CV, n0);
#pragma unroll
                for (int r = 0; r < 2; ++r)
                    *reinterpret_cast<float4*>(sdWV + (r0 + r) * CV + n0) =
                        make_float4(acc[r][0], acc[r][1], acc[r][2], acc[r][3]);
            } else if ((y -= t1) < t2) {
                const int r0 = 2 * (y / nk), n0 = 4 * (y - (y / nk) * nk);
                tile_mmk(acc, sdO, CV, r0, sS0T, KT, n0, V4);
#pragma unroll
                for (int r = 0; r < 2; ++r)
#pragma unroll
                    for (int cc = 0; cc < 4; ++cc) sdQp[r0 + r][n0 + cc] = acc[r][cc];
            } else if ((y -= t2) < t3) {
                const int r0 = 2 * (y / 4), n0 = 4 * (y % 4);
                tile_mmk(acc, sdO, CV, r0, sET, SR, n0, V4);
#pragma unroll
                for (int r = 0; r < 2; ++r)
#pragma unroll
                    for (int cc = 0; cc < 4; ++cc) sdM[r0 + r][n0 + cc] = n0 + cc <= r0 + r ? acc[r][cc] : 0.f;
            } else if ((y -= t3) < t4) {
                const int r0 = 2 * (y / nk), n0 = 4 * (y - (y / nk) * nk);
                tile_mmk(acc, sE, CV, r0, sdST, KT, n0, V4);
#pragma unroll
                for (int r = 0; r < 2; ++r)
#pragma unroll
                    for (int cc = 0; cc < 4; ++cc) sdWd[r0 + r][n0 + cc] = acc[r][cc];
            } else {
                const int i = y - t4;
                float sacc = 0.f;
                for (int jj = 0; jj < V; ++jj) sacc = fmaf(sS0T[jj * KT + i], sdST[jj * KT + i], sacc);
                sdPl[i] = sacc;
            }
        }
    }
    __syncthreads();
    // phase 2: dB = -dWV S0^T, dA = -strict_lower(dWV E^T); dv, d write
    {
        const int nk = K4 / 4;
        const int t1 = (CC / 2) * nk, t2 = (CC / 2) * (CC / 4);
        for (int x = tid; x < t1 + t2; x += GTH) {
            float acc[2][4] = {};
            if (x < t1) {
                const int r0 = 2 * (x / nk), n0 = 4 * (x - (x / nk) * nk);
                tile_mmk(acc, sdWV, CV, r0, sS0T, KT, n0, V4);
#pragma unroll
                for (int r = 0; r < 2; ++r)
#pragma unroll
                    for (int cc = 0; cc < 4; ++cc) sdB[r0 + r][n0 + cc] = -acc[r][cc];
            } else {
                const int y = x - t1, r0 = 2 * (y / 4), n0 = 4 * (y % 4);
                tile_mmk(acc, sdWV, CV, r0, sET, SR, n0, V4);
#pragma unroll
                for (int r = 0; r < 2; ++r)
#pragma unroll
                    for (int cc = 0; cc < 4; ++cc) sdA[r0 + r][n0 + cc] = n0 + cc < r0 + r ? -acc[r][cc] : 0.f;
            }
        }
        for (int x = tid; x < n * V; x += GTH) {
            const int t = x / V, j = x - t * V;
            const size_t gi = tok(p, b, t0 + t, h) * V + j;
            const float dwv = sact[t] ? sdWV[t * CV + j] : 0.f;
            p.dv[gi] = sact[t] ? dwv * p.write[gi] : 0.f;
            p.dwrite[gi] = sact[t] ? dwv * p.v[gi] : 0.f;
        }
    }
    __syncthreads();
    // phase 3, per (token t, key channel i): dq, d(ek), dk from A, M, Wd; dP
    for (int x = tid; x < CC * K; x += GTH) {
        const int t = x / K, i = x - t * K;
        const float pt = sP[t][i];
        float gq = sdQp[t][i] * pt, dek = sdB[t][i] * pt;
        float prod = 1.f;  // d[t][s]
        for (int s = t; s >= 0; --s) {
            if (s < t) prod *= sf[s + 1][i];
            const float kv = sk[s][i] * prod;
            gq = fmaf(sdM[t][s], kv, gq);
            if (s < t) dek = fmaf(sdA[t][s], kv, dek);
        }
        float gk = sdM[t][t] * sq[t][i];
        prod = 1.f;  // d[t2][t]
        for (int t2 = t + 1; t2 < CC; ++t2) {
            prod *= sf[t2][i];
            gk = fmaf(fmaf(sdA[t2][t], sek[t2][i], sdM[t2][t] * sq[t2][i]), prod, gk);
        }
        gk = fmaf(sdWd[t][i], prod, gk);
        sdP[t][i] = fmaf(sdQp[t][i], sq[t][i], sdB[t][i] * sek[t][i]) + (t == CC - 1 ? sdPl[i] : 0.f);
        if (t < n) {
            const size_t gi = tok(p, b, t0 + t, h) * K + i;
            if (sact[t]) {
                const float ksc = (sen[t] > 0.f && skn[t] > 0.f) ? sgs[t] * sen[t] / skn[t] : 0.f;
                p.dq[gi] = gq;
                p.dk[gi] = fmaf(ksc, sk[t][i], fmaf(dek, ser[t][i], gk));
                p.derase[gi] = dek * sk[t][i];
            } else {
                p.dq[gi] = p.dk[gi] = p.derase[gi] = 0.f;
            }
        }
    }
    __syncthreads();
    // phase 4: d alpha.  Y[t][u] = dP_t P_{u-1} + sum_{s<u} DD[t][s] d[u-1][s] obeys
    // Y[t][u + 1] = f_u Y[t][u] + DD[t][u] (Y[t][0] = dP_t), so the thread of (token t, channel i)
    // walks u upwards for Y and back down for the terms d[t][u] Y[t][u], which it leaves in
    // C[t][u][i] (in the shared memory of E .. dS_end, no longer read, where it fits); then
    // df_u = sum_{t>=u} C[t][u].
    float* sC = smem_g + L.C;  // [CC][CC][KMAX]
    for (int x = tid; x < CC * K; x += GTH) {
        const int t = x / K, i = x - t * K;
        const float ekt = sek[t][i], qt = sq[t][i];
        const float wl = t == CC - 1 ? 1.f : 0.f;
        float y[CC];
        y[0] = sdP[t][i];
#pragma unroll
        for (int u = 1; u < CC; ++u) {
            if (u <= t) {
                const int s0 = u - 1;
                const float dd = fmaf(sdA[t][s0], ekt, fmaf(sdM[t][s0], qt, wl * sdWd[s0][i])) * sk[s0][i];
                y[u] = fmaf(sf[s0][i], y[u - 1], dd);
            }
        }
        float dtu = 1.f;  // d[t][u]
#pragma unroll
        for (int u = CC - 1; u >= 0; --u) {
            if (u <= t) {
                sC[(t * CC + u) * KMAX + i] = dtu * y[u];
                dtu *= sf[u][i];
            }
        }
    }
    __syncthreads();
    for (int x = tid; x < n * K; x += GTH) {
        const int u = x / K, i = x - u * K;
        float df = 0.f;
        for (int t = u; t < CC; ++t) df += sC[(t * CC + u) * KMAX + i];
        p.dalpha[tok(p, b, t0 + u, h) * K + i] = (sact[u] && !srst[u]) ? df : 0.f;
    }
}

template <int KMAX, int VG>
int launch_rev(const CBwdParams& p, int ngroups, int NB, size_t smem, cudaStream_t st) {
    static std::atomic<uint64_t> attr_done{0};
    const int rc = once_per_device(attr_done, [] {
        return cuda_status(cudaFuncSetAttribute(chunk_bwd_rev_kernel<KMAX, VG>,
                                                cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024),
                           "chunk backward: shared memory attribute");
    });
    if (rc != DBL_OK) return rc;
    chunk_bwd_rev_kernel<KMAX, VG><<<(unsigned)((int64_t)p.B * p.H * ngroups), CTH, smem, st>>>(p, ngroups, NB);
    return launch_status("chunk_bwd_rev_kernel");
}

template <int KMAX>
int launch_grad(const CBwdParams& p, cudaStream_t st) {
    static std::atomic<uint64_t> attr_done{0};
    const int rc = once_per_device(attr_done, [] {
        return cuda_status(cudaFuncSetAttribute(chunk_bwd_grad_kernel<KMAX>,
                                                cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024),
                           "chunk backward: shared memory attribute");
    });
    if (rc != DBL_OK) return rc;
    const size_t smem = (size_t)grad_smem(KMAX, p.V).total * sizeof(float);
    chunk_bwd_grad_kernel<KMAX><<<(unsigned)((int64_t)p.B * p.H * p.nch), GTH, smem, st>>>(p);
    return launch_status("chunk_bwd_grad_kernel");
}

// Workspace carve-up of the chunked backward, in floats.
struct CBwdWs {
    size_t ck, fwd, edits, rev, dE, dSe, total;
};
CBwdWs cbwd_ws(const SeqParams& sp) {
    CBwdWs W{};
    const size_t bh = (size_t)sp.B * sp.H, nch = (size_t)(sp.T + CC - 1) / CC;
    auto up4 = [](size_t x) { return (x + 3) & ~(size_t)3; };  // every segment starts on 16 bytes
    size_t o = 0;
    W.ck = o; o += up4(bh * nch * sp.K * sp.V);
    W.fwd = o; o += up4(chunk_scan_workspace_floats(sp, true));
    W.edits = o; o += up4((size_t)sp.B * sp.T * sp.H * sp.V);
    W.rev = o; o += up4(bh * nch * rev_block(sp.K, sp.V).total);
    W.dE = o; o += up4(bh * nch * CC * sp.V);
    W.dSe = o; o += up4(bh * nch * sp.K * sp.V);
    W.total = o;
    return W;
}

}  // namespace

// The forward parameters of the training scan with f32 [B,T,H,W] inputs and valid/reset masks, no
// outputs: the shape test of the chunked backward and the forward it runs.
SeqParams chunk_backward_forward_params(int B, int T, int H, int K, int V, const float* q, const float* k,
                                        const float* v, const float* alpha, const float* erase, const float* write,
                                        const float* valid, const float* reset, const float* initial) {
    SeqParams sp{};
    sp.B = B;
    sp.T = T;
    sp.H = H;
    sp.K = K;
    sp.V = V;
    const int64_t dk[4] = {B, T, H, K};
    const int64_t dv[4] = {B, T, H, V};
    const int64_t z[4] = {0, 0, 0, 0};
    sp.q = q;
    sp.k = k;
    sp.v = v;
    resolve_strides(z, dk, 4, sp.qs);
    resolve_strides(z, dk, 4, sp.ks);
    resolve_strides(z, dv, 4, sp.vs);
    sp.gate_mode = 0;
    sp.alpha = alpha;
    sp.erase = erase;
    sp.write = write;
    resolve_strides(z, dk, 4, sp.as);
    resolve_strides(z, dk, 4, sp.es);
    resolve_strides(z, dv, 4, sp.ws);
    sp.scale = 1.f;
    sp.mask_mode = 1;
    sp.valid = valid;
    sp.reset = reset;
    sp.init_mode = initial ? 1 : 0;
    sp.initial = initial;
    return sp;
}

size_t chunk_backward_workspace_floats(const SeqParams& sp) { return cbwd_ws(sp).total; }

// Whether the backward of `sp` runs in chunked form: the chunked forward's widths (K <= 64,
// V <= 128, T >= 32, a zero or given initial state), at any number of sequence-heads.  Unlike the
// forward it replaces a token-sequential kernel that is slower at every size measured (T512,
// K32/V64: 64 rows 1.21 vs 0.45 ms chunked, 1024 rows 9.0 vs 4.0 ms; K64/V128: 256 rows 6.4 vs
// 3.7 ms).
bool chunk_backward_supported(const SeqParams& sp) {
    return sp.K <= 64 && sp.V <= CVMAX && sp.init_mode != 2 && sp.T >= 2 * CC;
}

namespace {

// The backward proper (pre, reverse, gradient kernels) given the forward's chunk-start states `ck`,
// chunk maps `fwd` and edits; its own buffers from `ws` (the carve-up of cbwd_ws).
int chunk_backward_core(const SeqParams& sp, const float* g_out, const float* g_fin, const float* g_score,
                        float* dq, float* dk, float* dv, float* dalpha, float* derase, float* dwrite,
                        float* dinitial, const float* ck, const float* fwd, const float* edits, float* ws,
                        cudaStream_t st) {
    const CBwdWs W = cbwd_ws(sp);
    CBwdParams p{};
    p.B = sp.B;
    p.T = sp.T;
    p.H = sp.H;
    p.K = sp.K;
    p.V = sp.V;
    p.nch = (sp.T + CC - 1) / CC;
    p.q = static_cast<const float*>(sp.q);
    p.k = static_cast<const float*>(sp.k);
    p.v = static_cast<const float*>(sp.v);
    p.alpha = sp.alpha;
    p.erase = sp.erase;
    p.write = sp.write;
    p.valid = sp.valid;
    p.reset = sp.reset;
    p.g_out = g_out;
    p.g_fin = g_fin;
    p.g_score = g_score;
    p.dq = dq;
    p.dk = dk;
    p.dv = dv;
    p.dalpha = dalpha;
    p.derase = derase;
    p.dwrite = dwrite;
    p.dinitial = dinitial;
    p.fwd = fwd;
    p.ck = ck;
    p.edits = edits;
    p.rev = ws + W.rev;
    p.dE = ws + W.dE;
    p.dSe = ws + W.dSe;
    const int64_t bh = (int64_t)p.B * p.H;
    const unsigned gchunks = (unsigned)(bh * p.nch);
    if (p.K <= 32) chunk_bwd_pre_kernel<32><<<gchunks, CTH, 0, st>>>(p);
    else chunk_bwd_pre_kernel<64><<<gchunks, CTH, 0, st>>>(p);
    int rc = launch_status("chunk_bwd_pre_kernel");
    if (rc != DBL_OK) return rc;
    const int VG = bh * ((p.V + 31) / 32) >= 148 ? 32 : 16;
    const int ngroups = (p.V + VG - 1) / VG;
    const int K4 = (p.K + 3) & ~3;
    const size_t bfl = (size_t)rev_block(p.K, p.V).sh + (CC + p.K) * VG;
    int NB = 4;
    while (NB > 2 && ((size_t)2 * K4 * VG + NB * bfl) * sizeof(float) > 227 * 1024) --NB;
    const size_t smem = ((size_t)2 * K4 * VG + NB * bfl) * sizeof(float);
    if (p.K <= 32) rc = VG == 16 ? launch_rev<32, 16>(p, ngroups, NB, smem, st) : launch_rev<32, 32>(p, ngroups, NB, smem, st);
    else rc = VG == 16 ? launch_rev<64, 16>(p, ngroups, NB, smem, st) : launch_rev<64, 32>(p, ngroups, NB, smem, st);
    if (rc != DBL_OK) return rc;
    return p.K <= 32 ? launch_grad<32>(p, st) : launch_grad<64>(p, st);
}

// The saved context: chunk-start states, chunk maps (laid out as if scores were requested, so the
// size does not depend on the forward's optional outputs), every token's edit; each segment on
// 16 bytes.
struct CtxLayout {
    size_t ck, fwd, edits, total;
};
CtxLayout ctx_layout(const SeqParams& sp) {
    auto up4 = [](size_t x) { return (x + 3) & ~(size_t)3; };
    SeqParams with_scores = sp;
    float dummy = 0.f;
    with_scores.scores = &dummy;
    const size_t bh = (size_t)sp.B * sp.H, nch = (size_t)(sp.T + CC - 1) / CC;
    CtxLayout C{};
    size_t o = 0;
    C.ck = o; o += up4(bh * nch * sp.K * sp.V);
    C.fwd = o; o += up4(chunk_scan_workspace_floats(with_scores, true));
    C.edits = o; o += up4((size_t)sp.B * sp.T * sp.H * sp.V);
    C.total = o;
    return C;
}

}  // namespace

// Runs the chunked backward for 16-token checkpoints (the caller checked chunk_backward_supported on
// `sp`); `ws` holds chunk_backward_workspace_floats(sp) floats.  The forward runs first, into `ws`.
int launch_chunk_backward(const SeqParams& sp, const float* g_out, const float* g_fin, const float* g_score,
                          float* dq, float* dk, float* dv, float* dalpha, float* derase, float* dwrite,
                          float* dinitial, float* ws, cudaStream_t st) {
    const CBwdWs W = cbwd_ws(sp);
    SeqParams fp = sp;
    fp.chunk_states = ws + W.ck;
    fp.edits = ws + W.edits;
    const int rc = launch_chunk_scan(fp, DBL_F32, st, ws + W.fwd, true);
    if (rc != DBL_OK) return rc;
    return chunk_backward_core(sp, g_out, g_fin, g_score, dq, dk, dv, dalpha, derase, dwrite, dinitial, ws + W.ck,
                               ws + W.fwd, ws + W.edits, ws, st);
}

size_t chunk_context_floats(const SeqParams& sp) { return ctx_layout(sp).total; }

// The forward of `sp` (outputs as requested) in chunked form, keeping its chunk-start states, maps
// and edits in `ctx`.
int launch_chunk_forward_saved(const SeqParams& sp, int in_dtype, float* ctx, cudaStream_t st) {
    const CtxLayout C = ctx_layout(sp);
    SeqParams fp = sp;
    fp.chunk_states = ctx + C.ck;
    fp.edits = ctx + C.edits;
    return launch_chunk_scan(fp, in_dtype, st, ctx + C.fwd, true);
}

// The backward from a context launch_chunk_forward_saved wrote for the same inputs.
int launch_chunk_backward_saved(const SeqParams& sp, const float* g_out, const float* g_fin, const float* g_score,
                                float* dq, float* dk, float* dv, float* dalpha, float* derase, float* dwrite,
                                float* dinitial, const float* ctx, float* ws, cudaStream_t st) {
    const CtxLayout C = ctx_layout(sp);
    return chunk_backward_core(sp, g_out, g_fin, g_score, dq, dk, dv, dalpha, derase, dwrite, dinitial, ctx + C.ck,
                               ctx + C.fwd, ctx + C.edits, ws, st);
}

}  // namespace dbl
