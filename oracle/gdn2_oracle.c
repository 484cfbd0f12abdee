/*
 * CPU oracle for the GDN-2 hot path (gated delta rule + relay merge).
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product path links, loads or calls this
 * file: only tests/, __graft_entry__.smoke() and the cpu_baseline / reference legs of
 * bench.py use it, and only as the checker or the timed CPU baseline.
 *
 * It restates, in plain C, the reference's CPU algorithms for the path:
 *
 *   orc_gdn2_scan_f64      crates/mixers/src/reference.rs:41-119   (f64 sequential oracle)
 *   orc_gdn2_doc_scan_f64  crates/mixers/src/gdn2_reference.rs:87-105 (inclusive doc limits)
 *   orc_gdn2_step_f64      crates/mixers/src/gdn2_reference.rs:52-83  (one recurrent step)
 *   orc_chunk_scan_f32     crates/mixers/src/chunk.rs:129-250 (chunkwise tensor solver,
 *                          the reference's CPU path; f32, OpenMP over batch x head)
 *   orc_relay_merge_f64    reuse/crates/dre-attention/src/oracle.rs:66-100 (one softmax over
 *                          concatenated key segments) with the [max, sum] statistics and the
 *                          empty-row convention of relay_attention_kernel.rs:113-128
 *   orc_relay_online_f32   reuse/crates/dre-attention/src/relay_attention_kernel.rs:63-111
 *                          (the online-softmax recurrence, in the kernel's f32 arithmetic)
 *   orc_relay_window_f64   relay_attention_kernel.rs:38-130 reference layout: +-radius
 *                          document window plus relay slots of the query's document
 *   orc_gdn_training_backward_f64  crates/kernels/src/gdn_training.rs:117-284 (the backward of
 *                          the stateful fused scan: gradients of q, k, v, gates and initial)
 *
 * Layouts (all contiguous, row-major):
 *   q, k, alpha, erase : [B,T,H,K]      v, write : [B,T,H,V]
 *   valid, reset       : [B,T] (nonzero = true)
 *   state / initial    : [B,H,K,V]  key-major, element (i,j) at i*V+j (reference.rs:53)
 *   out                : [B,T,H,V]      scores : [B,T,H]
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define IDX4(b, t, h, c, T, H, W) ((((size_t)(b) * (T) + (t)) * (H) + (h)) * (W) + (c))

/* ------------------------------------------------------------------------------------------
 * Sequential f64 scan.  Step order is exactly reference.rs:57-111:
 *   padding -> output 0, state unchanged, score 0;  reset -> state = 0;  S = diag(alpha) S;
 *   edit_j = write_j v_j - sum_i erase_i k_i S_ij;  score = |k| |edit|;
 *   S += k edit^T;  o_j = sum_i q_i S_ij.
 * Returns 0, or -1 on a non-finite input (reference.rs:58-61 panics there).
 * states_out (optional) receives the state after every token: [B,H,T,K,V].
 * ---------------------------------------------------------------------------------------- */
/* One (b, h) row of orc_gdn2_scan_f64; S and edit are K*V and V scratch doubles. */
static int scan_row_f64(int b, int h, int T, int H, int K, int V,
                        const double *q, const double *k, const double *v,
                        const double *alpha, const double *erase, const double *write,
                        const uint8_t *valid, const uint8_t *reset, const double *initial,
                        double *out, double *final_state, double *scores, double *states_out,
                        double *S, double *edit)
{
    const size_t sbase = ((size_t)b * H + h) * K * V;
    if (initial) memcpy(S, initial + sbase, sizeof(double) * K * V);
    else memset(S, 0, sizeof(double) * K * V);
    for (int t = 0; t < T; ++t) {
        const double *qt = q + IDX4(b, t, h, 0, T, H, K);
        const double *kt = k + IDX4(b, t, h, 0, T, H, K);
        const double *vt = v + IDX4(b, t, h, 0, T, H, V);
        const double *at = alpha + IDX4(b, t, h, 0, T, H, K);
        const double *et = erase + IDX4(b, t, h, 0, T, H, K);
        const double *wt = write + IDX4(b, t, h, 0, T, H, V);
        double *ot = out ? out + IDX4(b, t, h, 0, T, H, V) : NULL;
        for (int i = 0; i < K; ++i)
            if (!isfinite(qt[i]) || !isfinite(kt[i]) || !isfinite(at[i]) || !isfinite(et[i])) return -1;
        for (int j = 0; j < V; ++j)
            if (!isfinite(vt[j]) || !isfinite(wt[j])) return -1;
        const int act = valid ? valid[(size_t)b * T + t] != 0 : 1;
        const int rst = reset ? reset[(size_t)b * T + t] != 0 : 0;
        if (!act) {
            if (ot) memset(ot, 0, sizeof(double) * V);
            if (scores) scores[((size_t)b * T + t) * H + h] = 0.0;
        } else {
            if (rst) memset(S, 0, sizeof(double) * K * V);
            for (int i = 0; i < K; ++i)
                for (int j = 0; j < V; ++j) S[(size_t)i * V + j] *= at[i];
            for (int j = 0; j < V; ++j) {
                double e = wt[j] * vt[j];
                for (int i = 0; i < K; ++i) e -= et[i] * kt[i] * S[(size_t)i * V + j];
                edit[j] = e;
            }
            double kk = 0.0, ee = 0.0;
            for (int i = 0; i < K; ++i) kk += kt[i] * kt[i];
            for (int j = 0; j < V; ++j) ee += edit[j] * edit[j];
            if (scores) scores[((size_t)b * T + t) * H + h] = sqrt(kk * ee);
            if (ot) memset(ot, 0, sizeof(double) * V);
            for (int i = 0; i < K; ++i)
                for (int j = 0; j < V; ++j) {
                    S[(size_t)i * V + j] += kt[i] * edit[j];
                    if (ot) ot[j] += qt[i] * S[(size_t)i * V + j];
                }
        }
        if (states_out)
            memcpy(states_out + ((((size_t)b * H + h) * T + t) * K * V), S, sizeof(double) * K * V);
    }
    if (final_state) memcpy(final_state + sbase, S, sizeof(double) * K * V);
    return 0;
}

int orc_gdn2_scan_f64(int B, int T, int H, int K, int V,
                      const double *q, const double *k, const double *v,
                      const double *alpha, const double *erase, const double *write,
                      const uint8_t *valid, const uint8_t *reset, const double *initial,
                      double *out, double *final_state, double *scores, double *states_out)
{
    int status = 0;
    /* the (b, h) rows are independent: one row per OpenMP task, each with its own scratch */
#pragma omp parallel for schedule(dynamic, 1)
    for (int bh = 0; bh < B * H; ++bh) {
        double *edit = (double *)malloc(sizeof(double) * (size_t)V);
        double *S = (double *)malloc(sizeof(double) * (size_t)K * V);
        int rc = (!edit || !S) ? -2
                               : scan_row_f64(bh / H, bh % H, T, H, K, V, q, k, v, alpha, erase, write, valid,
                                              reset, initial, out, final_state, scores, states_out, S, edit);
        if (rc != 0) {
#pragma omp critical
            if (status == 0 || rc == -1) status = rc;
        }
        free(edit);
        free(S);
    }
    return status;
}

/* ------------------------------------------------------------------------------------------
 * gdn2_reference::scan (gdn2_reference.rs:87-105): inclusive limits, `end < start` is padding
 * (state snapshot kept, output 0), `start == t` resets.  Zero initial state.  Equivalent to the
 * sequential scan with valid = end >= start and reset = start == t.
 * ---------------------------------------------------------------------------------------- */
int orc_gdn2_doc_scan_f64(int B, int T, int H, int K, int V,
                          const double *q, const double *k, const double *v,
                          const double *alpha, const double *erase, const double *write,
                          const int32_t *doc_start, const int32_t *doc_end, double *out)
{
    uint8_t *valid = (uint8_t *)malloc((size_t)B * T);
    uint8_t *reset = (uint8_t *)malloc((size_t)B * T);
    if (!valid || !reset) { free(valid); free(reset); return -2; }
    for (int b = 0; b < B; ++b)
        for (int t = 0; t < T; ++t) {
            const size_t x = (size_t)b * T + t;
            valid[x] = doc_end[x] >= doc_start[x];
            reset[x] = doc_start[x] == t;
        }
    int rc = orc_gdn2_scan_f64(B, T, H, K, V, q, k, v, alpha, erase, write, valid, reset, NULL,
                               out, NULL, NULL, NULL);
    free(valid);
    free(reset);
    return rc;
}

/* ------------------------------------------------------------------------------------------
 * One recurrent step for N independent (sequence, head) states, in place
 * (gdn2_reference.rs:52-83, generalised to any K/V).  Layouts: q,k,alpha,erase [N,K];
 * v,write [N,V]; state [N,K,V]; out [N,V].
 * ---------------------------------------------------------------------------------------- */
int orc_gdn2_step_f64(int N, int K, int V, const double *q, const double *k, const double *v,
                      const double *alpha, const double *erase, const double *write,
                      double *state, double *out)
{
    double *read = (double *)malloc(sizeof(double) * (size_t)V);
    if (!read) return -2;
    for (int n = 0; n < N; ++n) {
        double *S = state + (size_t)n * K * V;
        const double *qn = q + (size_t)n * K, *kn = k + (size_t)n * K;
        const double *an = alpha + (size_t)n * K, *en = erase + (size_t)n * K;
        const double *vn = v + (size_t)n * V, *wn = write + (size_t)n * V;
        for (int i = 0; i < K; ++i)
            for (int j = 0; j < V; ++j) S[(size_t)i * V + j] *= an[i];
        for (int j = 0; j < V; ++j) {
            double r = 0.0;
            for (int i = 0; i < K; ++i) r += S[(size_t)i * V + j] * en[i] * kn[i];
            read[j] = wn[j] * vn[j] - r;
        }
        for (int i = 0; i < K; ++i)
            for (int j = 0; j < V; ++j) S[(size_t)i * V + j] += kn[i] * read[j];
        for (int j = 0; j < V; ++j) {
            double o = 0.0;
            for (int i = 0; i < K; ++i) o += S[(size_t)i * V + j] * qn[i];
            out[(size_t)n * V + j] = o;
        }
    }
    free(read);
    return 0;
}

/* ------------------------------------------------------------------------------------------
 * Chunkwise tensor solver, f32 (chunk.rs:129-250).  Per chunk, in the reference's order:
 *   mask q,k,v,erase,write by valid; alpha <- alpha (1-reset) valid + (1-valid)   (:155-169)
 *   prefix = cumprod(alpha)                                                         (:170)
 *   decay[r][s][i] = prod_{u=s+1..r} alpha_u[i], identity on r == s                 (:172-182)
 *   lower = strict_lower((erase k) decay k^T);  rhs = write v - (erase k prefix) S  (:184-194)
 *   inverse = sum_n (-lower)^n by repeated squaring                                (:211-220)
 *   edits = inverse rhs;  out = (q prefix) S + tril(q decay k^T) edits              (:221-227)
 *   scores = sqrt(|k|^2 |edit|^2) (0 at a zero edit);  S = prefix_C S + (tail k)^T edits.
 * chunk must be 1..=16 (chunk.rs:137-140).  OpenMP over batch x head with nthreads threads.
 * ---------------------------------------------------------------------------------------- */
int orc_chunk_scan_f32(int B, int T, int H, int K, int V,
                       const float *q, const float *k, const float *v,
                       const float *alpha, const float *erase, const float *write,
                       const float *valid, const float *reset, const float *initial, int chunk,
                       float *out, float *final_state, float *scores, int nthreads)
{
    if (chunk < 1 || chunk > 16) return -3;
    if (nthreads < 1) nthreads = 1;
    int failed = 0;
#pragma omp parallel for num_threads(nthreads) schedule(dynamic, 1)
    for (int bh = 0; bh < B * H; ++bh) {
        const int b = bh / H, h = bh % H;
        const int C = chunk;
        float *S = (float *)malloc(sizeof(float) * (size_t)K * V);
        float *mq = (float *)malloc(sizeof(float) * (size_t)C * K);
        float *mk = (float *)malloc(sizeof(float) * (size_t)C * K);
        float *me = (float *)malloc(sizeof(float) * (size_t)C * K);
        float *ma = (float *)malloc(sizeof(float) * (size_t)C * K);
        float *pre = (float *)malloc(sizeof(float) * (size_t)C * K);
        float *mv = (float *)malloc(sizeof(float) * (size_t)C * V);
        float *mw = (float *)malloc(sizeof(float) * (size_t)C * V);
        float *rhs = (float *)malloc(sizeof(float) * (size_t)C * V);
        float *ed = (float *)malloc(sizeof(float) * (size_t)C * V);
        float *dec = (float *)malloc(sizeof(float) * (size_t)C * C * K);
        float *low = (float *)malloc(sizeof(float) * (size_t)C * C);
        float *qk = (float *)malloc(sizeof(float) * (size_t)C * C);
        float *inv = (float *)malloc(sizeof(float) * (size_t)C * C);
        float *pw = (float *)malloc(sizeof(float) * (size_t)C * C);
        float *tmp = (float *)malloc(sizeof(float) * (size_t)C * C);
        float *act = (float *)malloc(sizeof(float) * (size_t)C);
        if (!S || !mq || !mk || !me || !ma || !pre || !mv || !mw || !rhs || !ed || !dec || !low ||
            !qk || !inv || !pw || !tmp || !act) {
#pragma omp atomic write
            failed = 1;
        } else {
            const size_t sbase = ((size_t)b * H + h) * K * V;
            if (initial) memcpy(S, initial + sbase, sizeof(float) * K * V);
            else memset(S, 0, sizeof(float) * K * V);
            for (int first = 0; first < T; first += C) {
                const int n = (T - first) < C ? (T - first) : C;
                for (int r = 0; r < n; ++r) {
                    const int t = first + r;
                    const float a = valid ? valid[(size_t)b * T + t] : 1.0f;
                    const float rs = reset ? reset[(size_t)b * T + t] : 0.0f;
                    act[r] = a;
                    for (int i = 0; i < K; ++i) {
                        const size_t x = IDX4(b, t, h, i, T, H, K);
                        mq[r * K + i] = q[x] * a;
                        mk[r * K + i] = k[x] * a;
                        me[r * K + i] = erase[x] * a;
                        ma[r * K + i] = alpha[x] * (1.0f - rs) * a + (1.0f - a);
                    }
                    for (int j = 0; j < V; ++j) {
                        const size_t x = IDX4(b, t, h, j, T, H, V);
                        mv[r * V + j] = v[x] * a;
                        mw[r * V + j] = write[x] * a;
                    }
                }
                for (int i = 0; i < K; ++i) {
                    float p = 1.0f;
                    for (int r = 0; r < n; ++r) { p *= ma[r * K + i]; pre[r * K + i] = p; }
                }
                /* decay[r][s][i], s <= r */
                for (int r = 0; r < n; ++r)
                    for (int s = 0; s <= r; ++s)
                        for (int i = 0; i < K; ++i) {
                            float p = 1.0f;
                            for (int u = s + 1; u <= r; ++u) p *= ma[u * K + i];
                            dec[((size_t)r * C + s) * K + i] = p;
                        }
                for (int r = 0; r < n; ++r)
                    for (int s = 0; s < n; ++s) {
                        float lo = 0.0f, qq = 0.0f;
                        if (s <= r)
                            for (int i = 0; i < K; ++i) {
                                const float f = dec[((size_t)r * C + s) * K + i] * mk[s * K + i];
                                lo += me[r * K + i] * mk[r * K + i] * f;
                                qq += mq[r * K + i] * f;
                            }
                        low[r * C + s] = (s < r) ? lo : 0.0f; /* tril(-1) */
                        qk[r * C + s] = (s <= r) ? qq : 0.0f; /* tril(0) */
                    }
                for (int r = 0; r < n; ++r)
                    for (int j = 0; j < V; ++j) {
                        float x = mw[r * V + j] * mv[r * V + j];
                        float sub = 0.0f;
                        for (int i = 0; i < K; ++i)
                            sub += me[r * K + i] * mk[r * K + i] * pre[r * K + i] * S[(size_t)i * V + j];
                        rhs[r * V + j] = x - sub;
                    }
                /* inverse = I; power = -lower; while covered < n: inverse += power inverse; ... */
                for (int r = 0; r < n; ++r)
                    for (int s = 0; s < n; ++s) {
                        inv[r * C + s] = (r == s) ? 1.0f : 0.0f;
                        pw[r * C + s] = -low[r * C + s];
                    }
                for (int covered = 1; covered < n;) {
                    for (int r = 0; r < n; ++r)
                        for (int s = 0; s < n; ++s) {
                            float acc = 0.0f;
                            for (int m = 0; m < n; ++m) acc += pw[r * C + m] * inv[m * C + s];
                            tmp[r * C + s] = inv[r * C + s] + acc;
                        }
                    memcpy(inv, tmp, sizeof(float) * C * C);
                    covered *= 2;
                    if (covered < n) {
                        for (int r = 0; r < n; ++r)
                            for (int s = 0; s < n; ++s) {
                                float acc = 0.0f;
                                for (int m = 0; m < n; ++m) acc += pw[r * C + m] * pw[m * C + s];
                                tmp[r * C + s] = acc;
                            }
                        memcpy(pw, tmp, sizeof(float) * C * C);
                    }
                }
                for (int r = 0; r < n; ++r)
                    for (int j = 0; j < V; ++j) {
                        float acc = 0.0f;
                        for (int s = 0; s < n; ++s) acc += inv[r * C + s] * rhs[s * V + j];
                        ed[r * V + j] = acc;
                    }
                for (int r = 0; r < n; ++r) {
                    const int t = first + r;
                    if (out)
                        for (int j = 0; j < V; ++j) {
                            float acc = 0.0f;
                            for (int i = 0; i < K; ++i)
                                acc += mq[r * K + i] * pre[r * K + i] * S[(size_t)i * V + j];
                            for (int s = 0; s <= r; ++s) acc += qk[r * C + s] * ed[s * V + j];
                            out[IDX4(b, t, h, j, T, H, V)] = acc;
                        }
                    if (scores) {
                        float kk = 0.0f, ee = 0.0f;
                        for (int i = 0; i < K; ++i) kk += mk[r * K + i] * mk[r * K + i];
                        for (int j = 0; j < V; ++j) ee += ed[r * V + j] * ed[r * V + j];
                        const float m2 = kk * ee;
                        scores[((size_t)b * T + t) * H + h] = (m2 == 0.0f) ? 0.0f : sqrtf(m2);
                    }
                }
                for (int i = 0; i < K; ++i) {
                    const float fd = pre[(n - 1) * K + i];
                    for (int j = 0; j < V; ++j) {
                        float acc = fd * S[(size_t)i * V + j];
                        for (int s = 0; s < n; ++s)
                            acc += dec[((size_t)(n - 1) * C + s) * K + i] * mk[s * K + i] * ed[s * V + j];
                        S[(size_t)i * V + j] = acc;
                    }
                }
            }
            if (final_state) memcpy(final_state + sbase, S, sizeof(float) * K * V);
        }
        free(S); free(mq); free(mk); free(me); free(ma); free(pre); free(mv); free(mw);
        free(rhs); free(ed); free(dec); free(low); free(qk); free(inv); free(pw); free(tmp);
        free(act);
    }
    return failed ? -2 : 0;
}

/* ------------------------------------------------------------------------------------------
 * Relay merge oracle: for each (sequence n, head h) one query attends, through ONE softmax,
 * to the concatenation [shared prefix keys ; the sequence's own keys] (oracle.rs:66-100 forms
 * attention over cat[local, relay] the same way).  Writes o, and the statistics of
 * relay_attention_kernel.rs:113-128: max = the largest eligible score, sum = sum exp(s - max).
 * A row with no eligible key writes o = 0, (max, sum) = (0, 1).
 * Layouts: q [N,H,D]; kp,vp [H,Lp,D]; ko,vo [N,H,Lo,D]; own_len [N] (NULL = Lo for all).
 * ---------------------------------------------------------------------------------------- */
int orc_relay_merge_f64(int N, int H, int D, int Lp, int Lo, const int32_t *own_len,
                        const double *q, const double *kp, const double *vp, const double *ko,
                        const double *vo, double scale, double *o, double *mx, double *sm)
{
    const int L = Lp + Lo;
    double *sc = (double *)malloc(sizeof(double) * (size_t)(L > 0 ? L : 1));
    if (!sc) return -2;
    for (int n = 0; n < N; ++n) {
        const int lo = own_len ? own_len[n] : Lo;
        if (lo < 0 || lo > Lo) { free(sc); return -3; }
        for (int h = 0; h < H; ++h) {
            const double *qq = q + ((size_t)n * H + h) * D;
            double *oo = o + ((size_t)n * H + h) * D;
            int cnt = 0;
            double m = 0.0;
            for (int p = 0; p < Lp; ++p) {
                const double *kk = kp + ((size_t)h * Lp + p) * D;
                double d = 0.0;
                for (int c = 0; c < D; ++c) d += qq[c] * kk[c];
                sc[cnt] = d * scale;
                if (cnt == 0 || sc[cnt] > m) m = sc[cnt];
                ++cnt;
            }
            for (int p = 0; p < lo; ++p) {
                const double *kk = ko + (((size_t)n * H + h) * Lo + p) * D;
                double d = 0.0;
                for (int c = 0; c < D; ++c) d += qq[c] * kk[c];
                sc[cnt] = d * scale;
                if (cnt == 0 || sc[cnt] > m) m = sc[cnt];
                ++cnt;
            }
            for (int c = 0; c < D; ++c) oo[c] = 0.0;
            if (cnt == 0) {
                mx[(size_t)n * H + h] = 0.0;
                sm[(size_t)n * H + h] = 1.0;
                continue;
            }
            double s = 0.0;
            for (int p = 0; p < cnt; ++p) {
                const double w = exp(sc[p] - m);
                const double *vv = (p < Lp) ? vp + ((size_t)h * Lp + p) * D
                                            : vo + (((size_t)n * H + h) * Lo + (p - Lp)) * D;
                for (int c = 0; c < D; ++c) oo[c] += w * vv[c];
                s += w;
            }
            for (int c = 0; c < D; ++c) oo[c] /= s;
            mx[(size_t)n * H + h] = m;
            sm[(size_t)n * H + h] = s;
        }
    }
    free(sc);
    return 0;
}

/* ------------------------------------------------------------------------------------------
 * The online-softmax recurrence of relay_attention_kernel.rs:73-111 in f32, over the same
 * concatenation as orc_relay_merge_f64 (prefix first, then own keys).  Used by the
 * known-answer tests: with one effective key the output is exactly that key's value, and with
 * L equal scores the normaliser is exactly L.
 *   next = (total == 0 || s > max) ? s : max;  a = total == 0 ? 0 : exp(max - next);
 *   p = exp(s - next);  total = total a + p;  acc = acc a + p v;  max = next.
 * ---------------------------------------------------------------------------------------- */
int orc_relay_online_f32(int N, int H, int D, int Lp, int Lo, const int32_t *own_len,
                         const float *q, const float *kp, const float *vp, const float *ko,
                         const float *vo, float scale, float *o, float *mx, float *sm)
{
    float *acc = (float *)malloc(sizeof(float) * (size_t)D);
    if (!acc) return -2;
    for (int n = 0; n < N; ++n) {
        const int lo = own_len ? own_len[n] : Lo;
        if (lo < 0 || lo > Lo) { free(acc); return -3; }
        for (int h = 0; h < H; ++h) {
            const float *qq = q + ((size_t)n * H + h) * D;
            float maximum = 0.0f, total = 0.0f;
            for (int c = 0; c < D; ++c) acc[c] = 0.0f;
            for (int p = 0; p < Lp + lo; ++p) {
                const float *kk = (p < Lp) ? kp + ((size_t)h * Lp + p) * D
                                           : ko + (((size_t)n * H + h) * Lo + (p - Lp)) * D;
                const float *vv = (p < Lp) ? vp + ((size_t)h * Lp + p) * D
                                           : vo + (((size_t)n * H + h) * Lo + (p - Lp)) * D;
                float dot = 0.0f;
                for (int c = 0; c < D; ++c) dot += qq[c] * kk[c];
                const float s = dot * scale;
                const float next = (total == 0.0f || s > maximum) ? s : maximum;
                const float a = (total == 0.0f) ? 0.0f : expf(maximum - next);
                const float pr = expf(s - next);
                total = total * a + pr;
                for (int c = 0; c < D; ++c) acc[c] = acc[c] * a + pr * vv[c];
                maximum = next;
            }
            float *oo = o + ((size_t)n * H + h) * D;
            if (Lp + lo == 0) {
                for (int c = 0; c < D; ++c) oo[c] = 0.0f;
                mx[(size_t)n * H + h] = 0.0f;
                sm[(size_t)n * H + h] = 1.0f;
            } else {
                for (int c = 0; c < D; ++c) oo[c] = acc[c] / total;
                mx[(size_t)n * H + h] = maximum;
                sm[(size_t)n * H + h] = total;
            }
        }
    }
    free(acc);
    return 0;
}

/* ------------------------------------------------------------------------------------------
 * Reference-layout relay attention forward (relay_attention_kernel.rs:38-130): query t of row
 * b attends to keys in [t - radius, t + radius] that lie inside its inclusive document limits
 * [doc_start, doc_end], then to the `slots` relay keys of its document doc_id.  Padding rows
 * (doc_end < doc_start) write o = 0 and (0, 1).  One softmax over the union (oracle.rs:66-100).
 * Layouts: q,k,v [B,H,T,D]; rk,rv [Ndoc,H,slots,D]; doc_* [B,T]; o [B,H,T,D]; norm [B,H,T,2].
 * ---------------------------------------------------------------------------------------- */
int orc_relay_window_f64(int B, int H, int T, int D, int ndoc, int slots, int radius,
                         const double *q, const double *k, const double *v, const double *rk,
                         const double *rv, const int32_t *doc_id, const int32_t *doc_start,
                         const int32_t *doc_end, double scale, double *o, double *norm)
{
    const int cap = 2 * radius + 1 + slots;
    double *sc = (double *)malloc(sizeof(double) * (size_t)cap);
    const double **vs = (const double **)malloc(sizeof(double *) * (size_t)cap);
    if (!sc || !vs) { free(sc); free(vs); return -2; }
    for (int b = 0; b < B; ++b)
        for (int h = 0; h < H; ++h)
            for (int t = 0; t < T; ++t) {
                const size_t row = ((size_t)b * H + h) * T + t;
                const double *qq = q + row * D;
                double *oo = o + row * D;
                const int st = doc_start[(size_t)b * T + t], en = doc_end[(size_t)b * T + t];
                for (int c = 0; c < D; ++c) oo[c] = 0.0;
                if (en < st) { norm[row * 2] = 0.0; norm[row * 2 + 1] = 1.0; continue; }
                const int doc = doc_id[(size_t)b * T + t];
                if (doc < 0 || doc >= ndoc) { free(sc); free(vs); return -3; }
                int cnt = 0;
                double m = 0.0;
                const int lo = t > radius ? t - radius : 0;
                const int hi = t + radius < T ? t + radius : T - 1;
                for (int key = lo; key <= hi; ++key) {
                    if (key < st || key > en) continue;
                    const double *kk = k + (((size_t)b * H + h) * T + key) * D;
                    double d = 0.0;
                    for (int c = 0; c < D; ++c) d += qq[c] * kk[c];
                    sc[cnt] = d * scale;
                    vs[cnt] = v + (((size_t)b * H + h) * T + key) * D;
                    if (cnt == 0 || sc[cnt] > m) m = sc[cnt];
                    ++cnt;
                }
                for (int s = 0; s < slots; ++s) {
                    const double *kk = rk + (((size_t)doc * H + h) * slots + s) * D;
                    double d = 0.0;
                    for (int c = 0; c < D; ++c) d += qq[c] * kk[c];
                    sc[cnt] = d * scale;
                    vs[cnt] = rv + (((size_t)doc * H + h) * slots + s) * D;
                    if (cnt == 0 || sc[cnt] > m) m = sc[cnt];
                    ++cnt;
                }
                if (cnt == 0) { norm[row * 2] = 0.0; norm[row * 2 + 1] = 1.0; continue; }
                double s = 0.0;
                for (int p = 0; p < cnt; ++p) {
                    const double w = exp(sc[p] - m);
                    for (int c = 0; c < D; ++c) oo[c] += w * vs[p][c];
                    s += w;
                }
                for (int c = 0; c < D; ++c) oo[c] /= s;
                norm[row * 2] = m;
                norm[row * 2 + 1] = s;
            }
    free(sc);
    free(vs);
    return 0;
}

/* ------------------------------------------------------------------------------------------
 * Backward (vector-Jacobian product) of the stateful fused scan, restating the reference's
 * backward kernel (crates/kernels/src/gdn_training.rs:117-284; op gdn_training_backward,
 * gdn_training_ops.rs:95-127) for the loss
 *     L = sum g_out . out + sum g_fin . final_state + sum g_score . scores.
 * Per token t, in reverse, with A = dL/dS after the token (starting from g_fin):
 *   padding: no gradient, A unchanged;
 *   dd_j   = g_score |k| edit_j / |edit| + sum_i k_i A_ij   (after A += q dy^T, dy = g_out[t]);
 *   bar    = reset ? 0 : alpha (.) S_prev;   dq_i = sum_j (bar + k_i edit_j) dy_j;
 *   dk_i   = sum_j (A_ij edit_j - erase_i bar_ij dd_j) + g_score |edit| k_i / |k|;
 *   de_i   = -sum_j k_i bar_ij dd_j;   dv_j = dd_j write_j;   dw_j = dd_j v_j;
 *   dbar   = A - erase (.) k dd^T;  reset: A = 0, d alpha = 0;  else d alpha_i = sum_j dbar_ij
 *            S_prev_ij and A = alpha (.) dbar.
 * The score terms are taken only when |k| > 0 and |edit| > 0, as the reference does.  The
 * reference replays each checkpoint chunk in f32; here every state is kept in f64, which the
 * chunking does not change.  dinitial (optional) receives A after token 0.
 * ---------------------------------------------------------------------------------------- */
int orc_gdn_training_backward_f64(int B, int T, int H, int K, int V,
                                  const double *q, const double *k, const double *v,
                                  const double *alpha, const double *erase, const double *write,
                                  const uint8_t *valid, const uint8_t *reset, const double *initial,
                                  const double *g_out, const double *g_fin, const double *g_score,
                                  double *dq, double *dk, double *dv, double *dalpha, double *derase,
                                  double *dwrite, double *dinitial)
{
    double *S = (double *)malloc(sizeof(double) * (size_t)(T + 1) * K * V);
    double *ed = (double *)malloc(sizeof(double) * (size_t)T * V);
    double *kn = (double *)malloc(sizeof(double) * (size_t)T);
    double *en = (double *)malloc(sizeof(double) * (size_t)T);
    double *A = (double *)malloc(sizeof(double) * (size_t)K * V);
    double *dd = (double *)malloc(sizeof(double) * (size_t)V);
    if (!S || !ed || !kn || !en || !A || !dd) {
        free(S); free(ed); free(kn); free(en); free(A); free(dd);
        return -2;
    }
    for (int b = 0; b < B; ++b)
        for (int h = 0; h < H; ++h) {
            const size_t sbase = ((size_t)b * H + h) * K * V;
            /* forward: every state S_t (before token t) and every token's edit and norms */
            if (initial) memcpy(S, initial + sbase, sizeof(double) * K * V);
            else memset(S, 0, sizeof(double) * K * V);
            for (int t = 0; t < T; ++t) {
                const double *St = S + (size_t)t * K * V;
                double *Sn = S + (size_t)(t + 1) * K * V;
                const int act = valid ? valid[(size_t)b * T + t] != 0 : 1;
                const int rst = reset ? reset[(size_t)b * T + t] != 0 : 0;
                const double *kt = k + IDX4(b, t, h, 0, T, H, K);
                const double *at = alpha + IDX4(b, t, h, 0, T, H, K);
                const double *et = erase + IDX4(b, t, h, 0, T, H, K);
                const double *vt = v + IDX4(b, t, h, 0, T, H, V);
                const double *wt = write + IDX4(b, t, h, 0, T, H, V);
                double *edt = ed + (size_t)t * V;
                if (!act) {
                    memcpy(Sn, St, sizeof(double) * K * V);
                    memset(edt, 0, sizeof(double) * V);
                    kn[t] = en[t] = 0.0;
                    continue;
                }
                double k2 = 0.0, e2 = 0.0;
                for (int i = 0; i < K; ++i) k2 += kt[i] * kt[i];
                for (int j = 0; j < V; ++j) {
                    double x = wt[j] * vt[j];
                    for (int i = 0; i < K; ++i) x -= et[i] * kt[i] * (rst ? 0.0 : at[i] * St[(size_t)i * V + j]);
                    edt[j] = x;
                    e2 += x * x;
                }
                for (int i = 0; i < K; ++i)
                    for (int j = 0; j < V; ++j)
                        Sn[(size_t)i * V + j] = (rst ? 0.0 : at[i] * St[(size_t)i * V + j]) + kt[i] * edt[j];
                kn[t] = sqrt(k2);
                en[t] = sqrt(e2);
            }
            /* reverse */
            if (g_fin) memcpy(A, g_fin + sbase, sizeof(double) * K * V);
            else memset(A, 0, sizeof(double) * K * V);
            for (int t = T - 1; t >= 0; --t) {
                double *dqt = dq + IDX4(b, t, h, 0, T, H, K), *dkt = dk + IDX4(b, t, h, 0, T, H, K);
                double *dat = dalpha + IDX4(b, t, h, 0, T, H, K), *det = derase + IDX4(b, t, h, 0, T, H, K);
                double *dvt = dv + IDX4(b, t, h, 0, T, H, V), *dwt = dwrite + IDX4(b, t, h, 0, T, H, V);
                for (int i = 0; i < K; ++i) dqt[i] = dkt[i] = dat[i] = det[i] = 0.0;
                for (int j = 0; j < V; ++j) dvt[j] = dwt[j] = 0.0;
                const int act = valid ? valid[(size_t)b * T + t] != 0 : 1;
                if (!act) continue;
                const int rst = reset ? reset[(size_t)b * T + t] != 0 : 0;
                const double *qt = q + IDX4(b, t, h, 0, T, H, K);
                const double *kt = k + IDX4(b, t, h, 0, T, H, K);
                const double *at = alpha + IDX4(b, t, h, 0, T, H, K);
                const double *et = erase + IDX4(b, t, h, 0, T, H, K);
                const double *vt = v + IDX4(b, t, h, 0, T, H, V);
                const double *wt = write + IDX4(b, t, h, 0, T, H, V);
                const double *dy = g_out + IDX4(b, t, h, 0, T, H, V);
                const double gs = g_score ? g_score[((size_t)b * T + t) * H + h] : 0.0;
                const double *St = S + (size_t)t * K * V;
                const double *edt = ed + (size_t)t * V;
                double key_scale = 0.0;
                const int norms = kn[t] > 0.0 && en[t] > 0.0;
                if (norms) key_scale = gs * en[t] / kn[t];
                for (int i = 0; i < K; ++i)
                    for (int j = 0; j < V; ++j) A[(size_t)i * V + j] += qt[i] * dy[j];
                for (int j = 0; j < V; ++j) {
                    double x = norms ? gs * kn[t] * edt[j] / en[t] : 0.0;
                    for (int i = 0; i < K; ++i) x += kt[i] * A[(size_t)i * V + j];
                    dd[j] = x;
                }
                for (int i = 0; i < K; ++i) {
                    double gq = 0.0, gk = 0.0, ga = 0.0, ge = 0.0;
                    for (int j = 0; j < V; ++j) {
                        const double prev = St[(size_t)i * V + j];
                        const double bar = rst ? 0.0 : at[i] * prev;
                        double *a = A + (size_t)i * V + j;
                        gq += (bar + kt[i] * edt[j]) * dy[j];
                        gk += *a * edt[j] - et[i] * bar * dd[j];
                        ge -= kt[i] * bar * dd[j];
                        const double dbar = *a - et[i] * kt[i] * dd[j];
                        if (rst) {
                            *a = 0.0;
                        } else {
                            ga += dbar * prev;
                            *a = at[i] * dbar;
                        }
                    }
                    dqt[i] = gq;
                    dkt[i] = gk + key_scale * kt[i];
                    dat[i] = ga;
                    det[i] = ge;
                }
                for (int j = 0; j < V; ++j) {
                    dvt[j] = dd[j] * wt[j];
                    dwt[j] = dd[j] * vt[j];
                }
            }
            if (dinitial) memcpy(dinitial + sbase, A, sizeof(double) * K * V);
        }
    free(S); free(ed); free(kn); free(en); free(A); free(dd);
    return 0;
}
