// Chunked GDN-2 scan for the reference's training widths: the stateful recurrence of
// scan_seq.cu (gdn_training.rs:12-115; gdn2.rs:23-283 for document limits) rewritten so that the
// work between chunk boundaries is state-independent and runs for every chunk at once.
//
// Within a chunk of C tokens, with per-channel step factors f_t = 0 at a reset, alpha_t for
// other valid tokens and 1 for padding, the cumulative decays P_t = f_0 ... f_t and the pairwise
// products d[t][s] = f_{s+1} ... f_t (formed directly, never as ratios of cumulative products),
// the state after token t is S_t = P_t (.) S_0 + sum_{s <= t} d[t][s] (.) k_s edit_s^T.  The edits
// solve the unit lower-triangular system (I + A) edit = WV - B S_0 with
//   A[t][s] = sum_i (erase k)_t,i d[t][s]_i k_s,i (s < t),   B[t] = (erase k)_t (.) P_t,
// so with Ti = (I + A)^-1, U0 = Ti WV and B' = Ti B, edit = U0 - B' S_0, and
//   o   = (Q' - M B') S_0 + M U0,   Q'[t] = q_t (.) P_t,  M[t][s] = sum_i q_t,i d[t][s]_i k_s,i (s <= t)
//   S_C = (diag(P_last) - Wd^T B') S_0 + Wd^T U0,   Wd[s] = d[last][s] (.) k_s.
// Padding tokens have no edit and no output (their rows of WV, B and the output maps are zero).
//
// chunk_prep_kernel: one CTA per (b, h, chunk) builds the chunk's maps Qe = Q' - M B', O0 = M U0,
//   B', U0, G = diag(P_last) - Wd^T B', H = Wd^T U0 and |k_t|.
// chunk_main_kernel: one CTA per (b, h, column group) walks the chunks with its state columns in
//   shared memory (the columns of S evolve independently): o = Qe S + O0, edit = U0 - B' S (for
//   the scores |k| |edit|), S <- G S + H.
#include "scan_chunk.cuh"
#include "scan_seq_params.cuh"

#include <algorithm>
#include <mutex>

namespace dbl {
namespace {

using namespace chunk;

template <int KMAX, typename T>
__global__ void __launch_bounds__(CTH) chunk_prep_kernel(const SeqParams p, float* ws, int extra) {
    constexpr int KPL = KMAX / 32;  // key channels per lane in the running products
    constexpr int WS = CC + 4;      // row stride of Wd^T (16-byte rows on distinct banks)
    __shared__ __align__(16) float sk[CC][KMAX], sq[CC][KMAX], sek[CC][KMAX], sf[CC][KMAX];
    __shared__ __align__(16) float sPB[CC][KMAX];  // P_t, then (once P is folded into B and Q) B'
    __shared__ __align__(16) float sWdT[KMAX][WS];
    __shared__ __align__(16) float swv[CC][CVMAX], sU0[CC][CVMAX];
    __shared__ __align__(16) float sA[CC][CC], sM[CC][CC], sTi[CC][CC];
    __shared__ float sPl[KMAX];
    __shared__ int sact[CC];
    const int K = p.K, V = p.V;
    const int K4 = (K + 3) & ~3, V4 = (V + 3) & ~3;
    const int nch = (p.T + CC - 1) / CC;
    const int c = blockIdx.x % nch, bh = blockIdx.x / nch, b = bh / p.H, h = bh - (bh / p.H) * p.H;
    const int t0 = c * CC, n = min(CC, p.T - t0);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const T* qb = static_cast<const T*>(p.q) + b * p.qs[0] + h * p.qs[2];
    const T* kb = static_cast<const T*>(p.k) + b * p.ks[0] + h * p.ks[2];
    const T* vb = static_cast<const T*>(p.v) + b * p.vs[0] + h * p.vs[2];
    const bool scalar = p.gate_mode == 1;

    // token masks: act (valid, in range), rst (reset)
    if (tid < CC) {
        const int t = t0 + tid;
        int act = 0, rst = 0;
        if (tid < n) {
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
        }
        sact[tid] = act | (rst << 1);
    }
    __syncthreads();
    // inputs: k, q (scaled; zero for padding, whose outputs are zero), step factors f, erase k (zero
    // for padding), write v (zero for padding).  f32 rows with unit channel stride, 16-byte aligned
    // (the training entry's contiguous tensors at K, V multiples of 4) are read four at a time.
    auto al16 = [](const void* ptr, int64_t s0, int64_t s1, int64_t s2) {
        return ((reinterpret_cast<uintptr_t>(ptr) & 15) | (s0 & 3) | (s1 & 3) | (s2 & 3)) == 0;
    };
    const bool vec_k = sizeof(T) == 4 && !scalar && (K & 3) == 0 && p.ks[3] == 1 && p.qs[3] == 1 && p.as[3] == 1 &&
                       p.es[3] == 1 && al16(p.k, p.ks[0], p.ks[1], p.ks[2]) && al16(p.q, p.qs[0], p.qs[1], p.qs[2]) &&
                       al16(p.alpha, p.as[0], p.as[1], p.as[2]) && al16(p.erase, p.es[0], p.es[1], p.es[2]);
    const bool vec_v = sizeof(T) == 4 && !scalar && !p.v_zero && (V & 3) == 0 && p.vs[3] == 1 && p.ws[3] == 1 &&
                       al16(p.v, p.vs[0], p.vs[1], p.vs[2]) && al16(p.write, p.ws[0], p.ws[1], p.ws[2]);
    if (vec_k) {
        for (int x = tid; x < CC * (KMAX / 4); x += CTH) {
            const int u = x / (KMAX / 4), i = 4 * (x - u * (KMAX / 4));
            const int t = t0 + u;
            const bool act = sact[u] & 1, rst = sact[u] & 2;
            float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), qv = kv, f = make_float4(1.f, 1.f, 1.f, 1.f), ek = kv;
            if (u < n && i < K) {
                kv = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(kb) + t * p.ks[1] + i);
                if (act) {
                    const float4 q4 = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(qb) + t * p.qs[1] + i);
                    const float4 a4 = *reinterpret_cast<const float4*>(
                        p.alpha + (size_t)b * p.as[0] + (size_t)t * p.as[1] + (size_t)h * p.as[2] + i);
                    const float4 e4 = *reinterpret_cast<const float4*>(
                        p.erase + (size_t)b * p.es[0] + (size_t)t * p.es[1] + (size_t)h * p.es[2] + i);
                    qv = make_float4(q4.x * p.scale, q4.y * p.scale, q4.z * p.scale, q4.w * p.scale);
                    f = rst ? make_float4(0.f, 0.f, 0.f, 0.f) : a4;
                    ek = make_float4(e4.x * kv.x, e4.y * kv.y, e4.z * kv.z, e4.w * kv.w);
                }
            }
            *reinterpret_cast<float4*>(&sk[u][i]) = kv;
            *reinterpret_cast<float4*>(&sq[u][i]) = qv;
            *reinterpret_cast<float4*>(&sf[u][i]) = f;
            *reinterpret_cast<float4*>(&sek[u][i]) = ek;
        }
    }
    for (int x = tid; x < (vec_k ? 0 : CC * KMAX); x += CTH) {
        const int u = x / KMAX, i = x - u * KMAX;
        const int t = t0 + u;
        const bool act = sact[u] & 1, rst = sact[u] & 2;
        float kv = 0.f, qv = 0.f, f = 1.f, ek = 0.f;
        if (u < n && i < K) {
            kv = to_f32(kb[t * p.ks[1] + i * p.ks[3]]);
            if (act) {
                qv = to_f32(qb[t * p.qs[1] + i * p.qs[3]]) * p.scale;
                float a, e;
                if (scalar) {
                    a = p.alpha[(size_t)b * p.as[0] + (size_t)t * p.as[1] + (size_t)h * p.as[2]];
                    e = p.erase[(size_t)b * p.es[0] + (size_t)t * p.es[1] + (size_t)h * p.es[2]];
                } else {
                    a = p.alpha[(size_t)b * p.as[0] + (size_t)t * p.as[1] + (size_t)h * p.as[2] + (size_t)i * p.as[3]];
                    e = p.erase[(size_t)b * p.es[0] + (size_t)t * p.es[1] + (size_t)h * p.es[2] + (size_t)i * p.es[3]];
                }
                f = rst ? 0.f : a;
                ek = e * kv;
            }
        }
        sk[u][i] = kv;
        sq[u][i] = qv;
        sf[u][i] = f;
        sek[u][i] = ek;
    }
    if (vec_v) {
        for (int x = tid; x < CC * (CVMAX / 4); x += CTH) {
            const int u = x / (CVMAX / 4), j = 4 * (x - u * (CVMAX / 4));
            const int t = t0 + u;
            float4 wv = make_float4(0.f, 0.f, 0.f, 0.f);
            if (j < V && u < n && (sact[u] & 1)) {
                const float4 v4 = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(vb) + t * p.vs[1] + j);
                const float4 w4 = *reinterpret_cast<const float4*>(
                    p.write + (size_t)b * p.ws[0] + (size_t)t * p.ws[1] + (size_t)h * p.ws[2] + j);
                wv = make_float4(w4.x * v4.x, w4.y * v4.y, w4.z * v4.z, w4.w * v4.w);
            }
            *reinterpret_cast<float4*>(&swv[u][j]) = wv;
        }
    }
    for (int x = tid; x < (vec_v ? 0 : CC * CVMAX); x += CTH) {
        const int u = x / CVMAX, j = x - u * CVMAX;
        const int t = t0 + u;
        float wv = 0.f;
        if (j < V && u < n && (sact[u] & 1)) {
            const float vv = p.v_zero ? 0.f : to_f32(vb[t * p.vs[1] + j * p.vs[3]]);
            const float w = scalar ? p.erase[(size_t)b * p.es[0] + (size_t)t * p.es[1] + (size_t)h * p.es[2]]
                                   : p.write[(size_t)b * p.ws[0] + (size_t)t * p.ws[1] + (size_t)h * p.ws[2] +
                                             (size_t)j * p.ws[3]];
            wv = w * vv;
        }
        swv[u][j] = wv;
    }
    __syncthreads();

    // Running products, one source per warp step: s = -1 gives the chunk-start decays P_t, a token
    // s >= 0 gives column s of A and M and row s of Wd.  Lane l holds channels l, l + 32; the 32 sums
    // of a source (A[t][s] and M[t][s] for t = 0..15) leave the lanes by one reduce-scatter (31
    // shuffles) after which lane l holds sum l.
    for (int s = warp - 1; s < CC; s += CTH / 32) {
        float prod[KPL];
#pragma unroll
        for (int e = 0; e < KPL; ++e) prod[e] = 1.f;
        float r[2 * CC];
#pragma unroll
        for (int t = 0; t < CC; ++t) {
            float aa = 0.f, mm = 0.f;
            if (t > s) {
#pragma unroll
                for (int e = 0; e < KPL; ++e) {
                    const int i = lane + 32 * e;
                    prod[e] *= sf[t][i];
                    if (s < 0) {
                        sPB[t][i] = prod[e];
                    } else {
                        const float dk = prod[e] * sk[s][i];
                        aa = fmaf(sek[t][i], dk, aa);
                        mm = fmaf(sq[t][i], dk, mm);
                    }
                }
            } else if (t == s) {
#pragma unroll
                for (int e = 0; e < KPL; ++e) mm = fmaf(sq[t][lane + 32 * e], sk[t][lane + 32 * e], mm);
            }
            r[t] = aa;
            r[CC + t] = mm;
        }
        if (s >= 0) {
#pragma unroll
            for (int e = 0; e < KPL; ++e) sWdT[lane + 32 * e][s] = prod[e] * sk[s][lane + 32 * e];
#pragma unroll
            for (int o = 16, half = CC; o > 0; o >>= 1, half >>= 1) {
                const bool up = lane & o;
#pragma unroll
                for (int x = 0; x < half; ++x) {
                    const float send = up ? r[x] : r[x + half];
                    const float keep = up ? r[x + half] : r[x];
                    r[x] = keep + __shfl_xor_sync(0xffffffffu, send, o);
                }
            }
            if (lane < CC) sA[lane][s] = r[0];
            else sM[lane - CC][s] = r[0];
        }
    }
    __syncthreads();
    if (warp == 0) {
        // Ti = (I + A)^-1 by right-looking substitution, lane = column: once row s is final it is
        // subtracted from every later row, so the dependent chain is 16 steps long
        float x[CC];
#pragma unroll
        for (int t = 0; t < CC; ++t) x[t] = t == lane ? 1.f : 0.f;
#pragma unroll
        for (int s = 0; s < CC; ++s) {
#pragma unroll
            for (int t = s + 1; t < CC; ++t) x[t] = fmaf(-sA[t][s], x[s], x[t]);
        }
        if (lane < CC) {
#pragma unroll
            for (int t = 0; t < CC; ++t) sTi[t][lane] = x[t];
        }
    } else {
        // fold the decays in: B[t] = (erase k)_t (.) P_t and Q'[t] = q_t (.) P_t, in place
        for (int x = tid - 32; x < CC * KMAX; x += CTH - 32) {
            const int t = x / KMAX, i = x - t * KMAX;
            const float pt = sPB[t][i];
            sek[t][i] *= pt;
            sq[t][i] *= pt;
            if (t == CC - 1) sPl[i] = pt;
        }
    }
    const ChunkBlock L = chunk_block(K, V, extra != 0);
    const int KP = L.kp;
    float* blk = ws + ((size_t)bh * nch + c) * L.total;
    if (extra) {
        // P, Wd (rows of KP, zero beyond K) and M for the backward; Q' and Ti follow below
        for (int x = tid; x < CC * KP; x += CTH) {
            const int t = x / KP, i = x - t * KP;
            blk[L.pp + x] = i < K ? sPB[t][i] : 0.f;
            blk[L.wd + x] = i < K ? sWdT[i][t] : 0.f;
        }
        for (int x = tid; x < CC * CC; x += CTH) blk[L.mm + x] = sM[x / CC][x % CC];
    }
    __syncthreads();
    // B' = Ti B and U0 = Ti WV (2 x 4 tiles; B' overwrites P, which is no longer read)
    {
        const int nb = K4 / 4, nu = V4 / 4;
        const int tb = (CC / 2) * nb, tu = (CC / 2) * nu;
        for (int x = tid; x < tb + tu; x += CTH) {
            float acc[2][4] = {};
            const bool isb = x < tb;
            const int y = isb ? x : x - tb, nn = isb ? nb : nu;
            const int r0 = 2 * (y / nn), n0 = 4 * (y - (y / nn) * nn);
            if (isb) tile_mm(acc, &sTi[0][0], CC, r0, &sek[0][0], KMAX, n0);
            else tile_mm(acc, &sTi[0][0], CC, r0, &swv[0][0], CVMAX, n0);
            float* dst = isb ? &sPB[0][0] : &sU0[0][0];
            const int ld = isb ? KMAX : CVMAX;
#pragma unroll
            for (int r = 0; r < 2; ++r)
                *reinterpret_cast<float4*>(dst + (r0 + r) * ld + n0) =
                    make_float4(acc[r][0], acc[r][1], acc[r][2], acc[r][3]);
        }
    }
    __syncthreads();
    // the chunk's maps, to the workspace: Qe = Q' - M B', O0 = M U0, G = diag(P_last) - Wd^T B',
    // H = Wd^T U0 (2 x 4 tiles), B' and U0 as computed, zero padding columns K4 .. KP of the rows
    // of Qe, B' and G, and |k_t|
    if (extra) {
        for (int x = tid; x < CC * KP; x += CTH) {
            const int t = x / KP, i = x - t * KP;
            blk[L.qp + x] = i < K ? sq[t][i] : 0.f;
        }
        for (int x = tid; x < CC * CC; x += CTH) blk[L.ti + x] = sTi[x / CC][x % CC];
    }
    {
        const int nk = K4 / 4, nv = V4 / 4, rk = (K + 1) / 2;
        const int tq = (CC / 2) * nk, to = (CC / 2) * nv, tg = rk * nk, th = rk * nv;
        const int tbp = CC * nk, tu0 = CC * nv, tpad = 2 * CC + K;
        const int total = tq + to + tg + th + tbp + tu0 + tpad;
        for (int x = tid; x < total; x += CTH) {
            int y = x;
            if (y < tq + to + tg + th) {
                // a product tile
                int kind, nn;
                if (y < tq) { kind = 0; nn = nk; }
                else if ((y -= tq) < to) { kind = 1; nn = nv; }
                else if ((y -= to) < tg) { kind = 2; nn = nk; }
                else { y -= tg; kind = 3; nn = nv; }
                const int r0 = 2 * (y / nn), n0 = 4 * (y - (y / nn) * nn);
                float acc[2][4] = {};
                if (kind == 0) tile_mm(acc, &sM[0][0], CC, r0, &sPB[0][0], KMAX, n0);
                else if (kind == 1) tile_mm(acc, &sM[0][0], CC, r0, &sU0[0][0], CVMAX, n0);
                else if (kind == 2) tile_mm(acc, &sWdT[0][0], WS, r0, &sPB[0][0], KMAX, n0);
                else tile_mm(acc, &sWdT[0][0], WS, r0, &sU0[0][0], CVMAX, n0);
                // rows of Qe and G (stride KP) are 16-byte aligned, rows of O0 and H (stride V) when
                // V is a multiple of 4: one float4 store per tile row there
                const bool v4 = (V & 3) == 0;
#pragma unroll
                for (int r = 0; r < 2; ++r) {
                    const int row = r0 + r;
                    float4 w;
                    if (kind == 0) {
                        w = make_float4(sq[row][n0] - acc[r][0], sq[row][n0 + 1] - acc[r][1],
                                        sq[row][n0 + 2] - acc[r][2], sq[row][n0 + 3] - acc[r][3]);
                        *reinterpret_cast<float4*>(blk + L.qe + row * KP + n0) = w;
                    } else if (kind == 2) {
                        if (row < K) {
                            w = make_float4((row == n0 ? sPl[row] : 0.f) - acc[r][0],
                                            (row == n0 + 1 ? sPl[row] : 0.f) - acc[r][1],
                                            (row == n0 + 2 ? sPl[row] : 0.f) - acc[r][2],
                                            (row == n0 + 3 ? sPl[row] : 0.f) - acc[r][3]);
                            *reinterpret_cast<float4*>(blk + L.g + row * KP + n0) = w;
                        }
                    } else if (kind == 1 || row < K) {
                        float* dst = blk + (kind == 1 ? L.o0 : L.hh) + row * V;
                        if (v4) {
                            *reinterpret_cast<float4*>(dst + n0) = make_float4(acc[r][0], acc[r][1], acc[r][2], acc[r][3]);
                        } else {
#pragma unroll
                            for (int cc = 0; cc < 4; ++cc)
                                if (n0 + cc < V) dst[n0 + cc] = acc[r][cc];
                        }
                    }
                }
            } else if ((y -= tq + to + tg + th) < tbp + tu0) {
                // copies of B' and U0
                if (y < tbp) {
                    const int t = y / nk, n0 = 4 * (y - t * nk);
                    *reinterpret_cast<float4*>(blk + L.bp + t * KP + n0) = lds4(&sPB[t][n0]);
                } else {
                    y -= tbp;
                    const int t = y / nv, n0 = 4 * (y - t * nv);
                    if ((V & 3) == 0) {
                        *reinterpret_cast<float4*>(blk + L.u0 + t * V + n0) = lds4(&sU0[t][n0]);
                    } else {
#pragma unroll
                        for (int cc = 0; cc < 4; ++cc)
                            if (n0 + cc < V) blk[L.u0 + t * V + n0 + cc] = sU0[t][n0 + cc];
                    }
                }
            } else {
                // zero columns K4 .. KP of a row of Qe, B' or G
                y -= tbp + tu0;
                const int off = y < CC ? L.qe + y * KP : y < 2 * CC ? L.bp + (y - CC) * KP : L.g + (y - 2 * CC) * KP;
                *reinterpret_cast<float4*>(blk + off + K4) = make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
    }
    if (warp == 0) {
        for (int t = 0; t < CC; ++t) {
            float kk = 0.f;
            for (int i = lane; i < K; i += 32) kk = fmaf(sk[t][i], sk[t][i], kk);
            kk = warp_sum(kk);
            if (lane == 0) blk[L.kn + t] = (sact[t] & 1) ? sqrtf(kk) : 0.f;
        }
    }
}

// The sequential pass: one CTA per (b, h, column group of VG = 16 or 32 columns), the group's state
// columns S [K4][VG + 4] in shared memory (double-buffered; K4 = K rounded up to 4, the extra rows
// zero), the chunk maps in a ring of NB buffers filled by cp.async NB - 1 chunks ahead, so that a
// chunk's L2 latency hides behind the compute of the chunks before it.  The 256 slots (rr, j) own
// column j, tokens rr + m RP and state rows rr + m RP.  With NTH = 512 threads (grids of one wave)
// the two 16-lane halves of a warp take the same slots and alternate blocks of four key channels
// (one shuffle joins them; the state row stride VG + 4 puts the halves' rows on different banks);
// with 256 (more CTAs than SMs at key widths up to 32, where two CTAs share an SM) each slot is one
// thread.  One pass over the key channels
// accumulates o, the edit and the new state from the same state loads; one barrier per chunk; the
// scores of a chunk are written after the next chunk's barrier.  With one group the scores are final
// here; with several, each group writes its partial sums of edit^2 to `part`.
template <int KMAX, int VG, int NTH>
__global__ void __launch_bounds__(NTH) chunk_main_kernel(const SeqParams p, const float* ws, float* part,
                                                         int ngroups, int NB, int extra) {
    constexpr int MTH = NTH;
    constexpr int HALVES = NTH / 256;  // threads per slot
    constexpr int RP = 256 / VG;  // token (and state) rows per pass
    constexpr int NT = CC / RP;   // tokens per thread
    constexpr int NS = KMAX / RP; // state rows per thread
    constexpr int NP = VG / 16;   // 16-lane groups sharing one token
    constexpr int SST = VG + 4;   // state row stride
    constexpr int MAXCOL = ((2 * CC + KMAX) * VG + NTH - 1) / NTH;  // column-part copies per thread
    extern __shared__ __align__(16) float smain[];
    const int K = p.K, V = p.V, K4 = (K + 3) & ~3;
    const int nch = (p.T + CC - 1) / CC;
    const int grp = blockIdx.x % ngroups, bh = blockIdx.x / ngroups;
    const int b = bh / p.H, h = bh - (bh / p.H) * p.H;
    const int c0 = grp * VG, vg = min(VG, V - c0);
    const int tid = threadIdx.x, lane = tid & 31, half = HALVES == 2 ? lane >> 4 : 0;
    const int slot = HALVES == 2 ? (tid >> 5) * 16 + (lane & 15) : tid;
    const int j = slot % VG, rr = slot / VG;
    const ChunkBlock L = chunk_block(K, V, extra != 0);
    const int KP = L.kp;
    const int rows = 2 * CC + K;  // O0, U0, H rows
    const int bfl = L.sh + rows * VG;
    float* Sb0 = smain;
    float* Sb1 = smain + K4 * SST;
    float* bb0 = smain + 2 * K4 * SST;  // NB buffers of bfl floats
    float* ssqp = bb0 + NB * bfl;       // [2][CC][NP]
    const bool vec = (V & 3) == 0;
    const size_t sbase = ((size_t)b * p.H + h) * K * V;
    for (int x = tid; x < K4 * SST; x += MTH) {
        const int i = x / SST, jj = x - i * SST;
        Sb0[x] = (p.init_mode == 1 && i < K && jj < vg) ? p.initial[sbase + (size_t)i * V + c0 + jj] : 0.f;
        Sb1[x] = 0.f;
    }
    // this thread's copies of the column-sliced part (O0, U0, H rows), the same every chunk:
    // shared-memory and block offsets in floats (16-byte copies when V is a multiple of 4)
    int soff[MAXCOL], goff[MAXCOL];
    const int per = vec ? vg >> 2 : vg, ncopy = rows * per;
#pragma unroll
    for (int k = 0; k < MAXCOL; ++k) {
        const int x = tid + k * MTH;
        const int r = x / per, w = x - r * per;
        soff[k] = L.sh + r * VG + (vec ? 4 * w : w);
        goff[k] = L.sh + r * V + c0 + (vec ? 4 * w : w);
    }
    // stages chunk c into buffer `buf` and commits one group (an empty one past the last chunk)
    auto prefetch = [&](int c, int buf) {
        if (c < nch) {
            const float* src = ws + ((size_t)bh * nch + c) * L.total;
            float* dst = bb0 + buf * bfl;
            for (int x = tid; x < L.sh / 4; x += MTH) cp_async16(dst + 4 * x, src + 4 * x);
#pragma unroll
            for (int k = 0; k < MAXCOL; ++k) {
                if (tid + k * MTH >= ncopy) break;  // a thread's copies are a prefix of the slots
                if (vec) cp_async16(dst + soff[k], src + goff[k]);
                else cp_async4(dst + soff[k], src + goff[k]);
            }
        }
        cp_async_commit();
    };
    auto write_scores = [&](int c, float kn) {
        const int t0 = c * CC, n = min(CC, p.T - t0);
        if (tid < n) {
            const float* sp = ssqp + (c & 1) * CC * NP + tid * NP;
            float s = 0.f;
#pragma unroll
            for (int w = 0; w < NP; ++w) s += sp[w];
            const size_t si = ((size_t)b * p.T + t0 + tid) * p.H + h;
            if (ngroups == 1) p.scores[si] = kn * sqrtf(s);
            else part[(size_t)grp * p.B * p.T * p.H + si] = s;
        }
    };
    for (int c = 0; c < NB - 1; ++c) prefetch(c, c);
    // this thread's output and edit offsets at token 0
    const size_t out_base = (size_t)b * p.os[0] + (size_t)h * p.os[2] + (size_t)(c0 + j) * p.os[3];
    const size_t edit_base = ((size_t)b * p.T * p.H + h) * V + c0 + j;
    float kn_prev = 0.f;
    int cur = 0;  // buffer of chunk c; chunk c + NB - 1 goes to the buffer before it
    for (int c = 0; c < nch; ++c) {
        const int t0 = c * CC, n = min(CC, p.T - t0);
        cp_async_wait_pending(NB - 2);
        __syncthreads();  // chunk c's maps, the state and the previous chunk's edit sums are in place
        prefetch(c + NB - 1, cur == 0 ? NB - 1 : cur - 1);  // the buffer of chunk c - 1, finished by all
        const float* blk = bb0 + cur * bfl;
        cur = cur + 1 == NB ? 0 : cur + 1;
        if (p.scores && c > 0) write_scores(c - 1, kn_prev);
        const float* S = (c & 1) ? Sb1 : Sb0;
        float* Sn = (c & 1) ? Sb0 : Sb1;
        if (p.chunk_states && half == HALVES - 1 && j < vg) {
            float* cs = p.chunk_states + ((size_t)bh * nch + c) * K * V + c0 + j;
#pragma unroll
            for (int m = 0; m < NS; ++m)
                if (rr + m * RP < K) cs[(size_t)(rr + m * RP) * V] = S[(rr + m * RP) * SST + j];
        }
        kn_prev = (p.scores && tid < n) ? blk[L.kn + tid] : 0.f;
        const float* qe = blk + L.qe;
        const float* bp = blk + L.bp;
        const float* g = blk + L.g;
        const float* o0 = blk + L.sh;
        const float* u0 = o0 + CC * VG;
        const float* hh = u0 + CC * VG;
        // half 0 starts from the chunk's constant terms, half 1 from zero
        float o[NT], u[NT], acc[NS];
#pragma unroll
        for (int m = 0; m < NT; ++m) {
            o[m] = half ? 0.f : o0[(rr + m * RP) * VG + j];
            u[m] = half ? 0.f : u0[(rr + m * RP) * VG + j];
        }
#pragma unroll
        for (int m = 0; m < NS; ++m) acc[m] = (half == 0 && rr + m * RP < K) ? hh[(rr + m * RP) * VG + j] : 0.f;
        // unrolled over the compile-time key bound (K4 <= KMAX) so that the loads issue early
#pragma unroll
        for (int i0 = 0; i0 < KMAX; i0 += 4 * HALVES) {
            const int i = i0 + 4 * half;
            if (i >= K4) break;
            const float s0 = S[(i + 0) * SST + j], s1 = S[(i + 1) * SST + j];
            const float s2 = S[(i + 2) * SST + j], s3 = S[(i + 3) * SST + j];
#pragma unroll
            for (int m = 0; m < NT; ++m) {
                const float4 qv = lds4(qe + (rr + m * RP) * KP + i);
                const float4 bv = lds4(bp + (rr + m * RP) * KP + i);
                o[m] = fmaf(qv.x, s0, fmaf(qv.y, s1, fmaf(qv.z, s2, fmaf(qv.w, s3, o[m]))));
                u[m] = fmaf(-bv.x, s0, fmaf(-bv.y, s1, fmaf(-bv.z, s2, fmaf(-bv.w, s3, u[m]))));
            }
#pragma unroll
            for (int m = 0; m < NS; ++m) {
                if (rr + m * RP < K) {
                    const float4 gv = lds4(g + (rr + m * RP) * KP + i);
                    acc[m] = fmaf(gv.x, s0, fmaf(gv.y, s1, fmaf(gv.z, s2, fmaf(gv.w, s3, acc[m]))));
                }
            }
        }
        if constexpr (HALVES == 2) {
#pragma unroll
            for (int m = 0; m < NT; ++m) {
                o[m] += __shfl_xor_sync(0xffffffffu, o[m], 16);
                u[m] += __shfl_xor_sync(0xffffffffu, u[m], 16);
            }
#pragma unroll
            for (int m = 0; m < NS; ++m) acc[m] += __shfl_xor_sync(0xffffffffu, acc[m], 16);
        }
        if (half == HALVES - 1) {
#pragma unroll
            for (int m = 0; m < NS; ++m)
                if (rr + m * RP < K) Sn[(rr + m * RP) * SST + j] = acc[m];
        }
#pragma unroll
        for (int m = 0; m < NT; ++m) {
            const int t = rr + m * RP;
            if (half == 0 && t < n && j < vg) {
                if (p.edits) p.edits[edit_base + (size_t)(t0 + t) * p.H * V] = u[m];
                if (p.out) {
                    const size_t oi = out_base + (size_t)(t0 + t) * p.os[1];
                    if (p.out_dtype == DBL_BF16) static_cast<__nv_bfloat16*>(p.out)[oi] = __float2bfloat16_rn(o[m]);
                    else static_cast<float*>(p.out)[oi] = o[m];
                }
            }
            if (p.scores) {
                float e2 = j < vg ? u[m] * u[m] : 0.f;
#pragma unroll
                for (int w = 8; w > 0; w >>= 1) e2 += __shfl_xor_sync(0xffffffffu, e2, w);
                if (half == 0 && (lane & 15) == 0) ssqp[(c & 1) * CC * NP + t * NP + j / 16] = e2;
            }
        }
    }
    __syncthreads();
    if (p.scores) write_scores(nch - 1, kn_prev);
    if (p.final_state) {
        const float* S = (nch & 1) ? Sb1 : Sb0;
        for (int x = tid; x < K * vg; x += MTH) {
            const int i = x / vg, jj = x - i * vg;
            p.final_state[sbase + (size_t)i * V + c0 + jj] = S[i * SST + jj];
        }
    }
}

// scores = |k_t| sqrt(sum over column groups of the partial edit^2 sums)
__global__ void chunk_scores_kernel(const SeqParams p, const float* ws, const float* part, int ngroups, int extra) {
    const size_t n = (size_t)p.B * p.T * p.H;
    const size_t si = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (si >= n) return;
    const int h = (int)(si % p.H), t = (int)((si / p.H) % p.T), b = (int)(si / ((size_t)p.H * p.T));
    const int nch = (p.T + CC - 1) / CC;
    const ChunkBlock L = chunk_block(p.K, p.V, extra != 0);
    const float kn = ws[(((size_t)b * p.H + h) * nch + t / CC) * L.total + L.kn + t % CC];
    float s = 0.f;
    for (int g = 0; g < ngroups; ++g) s += part[(size_t)g * n + si];
    p.scores[si] = kn * sqrtf(s);
}
}  // namespace

// Whether the chunked path takes these shapes: key width <= 64, value width <= 128, a zero or given
// initial state (not the identity of span transitions), at least two chunks, and
// B*H*ceil(K/32)*ceil(V/64) <= 384.  Beyond that the token-sequential kernel has enough (b, h) rows
// to fill the GPU and does less work per token (measured at T512: K32/V64 96 rows 0.31 ms sequential
// vs 0.20 ms chunked, 128 rows 0.34 vs 0.22, 256 rows 0.42 vs 0.43; K64/V128 96 rows 0.60 vs 0.53;
// 512 rows 0.69 ms sequential).
bool chunk_scan_supported(const SeqParams& p) {
    return p.K <= 64 && p.V <= CVMAX && p.init_mode != 2 && p.T >= 2 * CC &&
           (int64_t)p.B * p.H * ((p.K + 31) / 32) * ((p.V + 63) / 64) <= 384;
}

// A stream-ordered pool per device for the chunk maps, created on first use; freed blocks stay in the
// pool (release threshold: never) so that repeated calls reuse them without driver allocations.
int scratch_pool(cudaMemPool_t* out) {
    static std::mutex mu;
    static cudaMemPool_t pools[64] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_status(e, "cudaGetDevice");
    if (dev < 0 || dev >= 64) return fail(DBL_ERR_UNSUPPORTED, "device ordinal %d out of range", dev);
    std::lock_guard<std::mutex> lock(mu);
    if (!pools[dev]) {
        cudaMemPoolProps props{};
        props.allocType = cudaMemAllocationTypePinned;
        props.location.type = cudaMemLocationTypeDevice;
        props.location.id = dev;
        cudaMemPool_t pool = nullptr;
        e = cudaMemPoolCreate(&pool, &props);
        if (e != cudaSuccess) return cuda_status(e, "chunk scan: cudaMemPoolCreate");
        uint64_t keep = ~uint64_t(0);
        e = cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep);
        if (e != cudaSuccess) return cuda_status(e, "chunk scan: pool release threshold");
        pools[dev] = pool;
    }
    *out = pools[dev];
    return DBL_OK;
}

namespace {

template <int KMAX, int VG, int NTH>
int launch_main_t(const SeqParams& p, const float* ws, float* part, int ngroups, int NB, int extra, size_t smem,
                  cudaStream_t st) {
    static std::atomic<uint64_t> attr_done{0};
    const int rc = once_per_device(attr_done, [] {
        return cuda_status(cudaFuncSetAttribute(chunk_main_kernel<KMAX, VG, NTH>,
                                                cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024),
                           "chunk scan: shared memory attribute");
    });
    if (rc != DBL_OK) return rc;
    chunk_main_kernel<KMAX, VG, NTH><<<(unsigned)((int64_t)p.B * p.H * ngroups), NTH, smem, st>>>(p, ws, part, ngroups, NB, extra);
    return launch_status("chunk_main_kernel");
}

// 512 threads when the grid is one wave of one CTA per SM or the key width is above 32 (the split
// of the key channels pays for the second wave: B8/T512/H4/K64/V128, 256 CTAs, 0.246 vs 0.270 ms),
// else 256 (two CTAs share an SM: B4/T512/H16/K32/V128, 256 CTAs, 0.215 vs 0.264 ms)
template <int KMAX, int VG>
int launch_main(const SeqParams& p, const float* ws, float* part, int ngroups, int NB, int extra, size_t smem,
                cudaStream_t st) {
    if ((int64_t)p.B * p.H * ngroups <= 148 || p.K > 32)
        return launch_main_t<KMAX, VG, 512>(p, ws, part, ngroups, NB, extra, smem, st);
    return launch_main_t<KMAX, VG, 256>(p, ws, part, ngroups, NB, extra, smem, st);
}

template <int KMAX>
int launch_main_vg(const SeqParams& p, const float* ws, float* part, int VG, int ngroups, int NB, int extra,
                   size_t smem, cudaStream_t st) {
    if (VG == 16) return launch_main<KMAX, 16>(p, ws, part, ngroups, NB, extra, smem, st);
    return launch_main<KMAX, 32>(p, ws, part, ngroups, NB, extra, smem, st);
}

}  // namespace

// Floats of the chunk maps (and partial score sums) a chunked scan of `p` uses; with `extra` the
// maps the backward keeps as well.
size_t chunk_scan_workspace_floats(const SeqParams& p, bool extra) {
    const int nch = (p.T + CC - 1) / CC;
    const int64_t bh = (int64_t)p.B * p.H;
    const int VG = bh * ((p.V + 31) / 32) >= 148 ? 32 : 16;
    const int ngroups = (p.V + VG - 1) / VG;
    const size_t part = (p.scores && ngroups > 1) ? (size_t)ngroups * bh * p.T : 0;
    return (size_t)bh * nch * chunk_block(p.K, p.V, extra).total + part;
}

// Runs the chunked scan: chunk maps (and partial score sums) in `ext_ws` when given (it must hold
// chunk_scan_workspace_floats(p, extra) floats and outlive the launches), else in a workspace from
// the library's stream-ordered pool, released on the stream after the last kernel.
int launch_chunk_scan(const SeqParams& p, int in_dtype, cudaStream_t st, float* ext_ws, bool extra) {
    const int nch = (p.T + CC - 1) / CC;
    const ChunkBlock L = chunk_block(p.K, p.V, extra);
    const int64_t bh = (int64_t)p.B * p.H;
    // column groups of 32 columns when that still gives a full wave of CTAs, else of 16
    const int VG = bh * ((p.V + 31) / 32) >= 148 ? 32 : 16;
    const int ngroups = (p.V + VG - 1) / VG;
    if (bh * nch > 0x7fffffffLL || bh * ngroups > 0x7fffffffLL)
        return fail(DBL_ERR_UNSUPPORTED, "chunk scan: grid exceeds 32-bit limits");
    const size_t ws_floats = (size_t)bh * nch * L.total;
    const size_t part_floats = (p.scores && ngroups > 1) ? (size_t)ngroups * bh * p.T : 0;
    float* ws = ext_ws;
    int rc = DBL_OK;
    if (!ws) {
        // while `st` is being captured into a CUDA graph the allocation becomes a graph memory node
        // (cudaMallocAsync); otherwise it comes from the library's pool
        cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
        cudaError_t e = cudaStreamIsCapturing(st, &cap);
        if (e != cudaSuccess) return cuda_status(e, "chunk scan: cudaStreamIsCapturing");
        const size_t bytes = (ws_floats + part_floats) * sizeof(float);
        if (cap == cudaStreamCaptureStatusActive) {
            e = cudaMallocAsync(reinterpret_cast<void**>(&ws), bytes, st);
        } else {
            cudaMemPool_t pool = nullptr;
            rc = scratch_pool(&pool);
            if (rc != DBL_OK) return rc;
            e = cudaMallocFromPoolAsync(reinterpret_cast<void**>(&ws), bytes, pool, st);
        }
        if (e != cudaSuccess) return cuda_status(e, "chunk scan: workspace");
    }
    float* part = ws + ws_floats;
    const bool bf = in_dtype == DBL_BF16;
    const unsigned gprep = (unsigned)(bh * nch);
    const int ex = extra ? 1 : 0;
    if (p.K <= 32) {
        if (bf) chunk_prep_kernel<32, __nv_bfloat16><<<gprep, CTH, 0, st>>>(p, ws, ex);
        else chunk_prep_kernel<32, float><<<gprep, CTH, 0, st>>>(p, ws, ex);
    } else {
        if (bf) chunk_prep_kernel<64, __nv_bfloat16><<<gprep, CTH, 0, st>>>(p, ws, ex);
        else chunk_prep_kernel<64, float><<<gprep, CTH, 0, st>>>(p, ws, ex);
    }
    rc = launch_status("chunk_prep_kernel");
    if (rc == DBL_OK) {
        const int K4 = (p.K + 3) & ~3;
        const int np = VG / 16;
        const size_t sfl = (size_t)2 * K4 * (VG + 4);  // the two state buffers
        const size_t bfl = (size_t)L.sh + (2 * CC + p.K) * VG;
        // the deepest ring of 4, 3 or 2 chunk buffers that fits in 227 KB
        int NB = 4;
        while (NB > 2 && (sfl + NB * bfl + 2 * CC * np) * sizeof(float) > 227 * 1024) --NB;
        const size_t smem = (sfl + NB * bfl + 2 * CC * np) * sizeof(float);
        rc = p.K <= 32 ? launch_main_vg<32>(p, ws, part, VG, ngroups, NB, ex, smem, st)
                       : launch_main_vg<64>(p, ws, part, VG, ngroups, NB, ex, smem, st);
    }
    if (rc == DBL_OK && part_floats) {
        const size_t n = (size_t)bh * p.T;
        chunk_scores_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(p, ws, part, ngroups, ex);
        rc = launch_status("chunk_scores_kernel");
    }
    if (!ext_ws) {
        const cudaError_t ef = cudaFreeAsync(ws, st);
        if (rc == DBL_OK) rc = cuda_status(ef, "chunk scan: workspace release");
    }
    return rc;
}

}  // namespace dbl
