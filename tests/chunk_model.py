"""numpy model of the tensor-core prefill kernel's arithmetic (prefill_tc.cu), for CPU tests.

It follows the kernel step by step -- log-space decay products with reset counting, the blocked
16 x 16 inverse of (I + A), and bf16 rounding exactly where the kernel rounds an MMA operand
(S, T and Delta to one bf16; R and P to a bf16 hi + lo pair) -- so the numerical error budget of
the kernel can be checked against the oracle without a GPU.  Test infrastructure only.
"""
from __future__ import annotations

import numpy as np

from fixtures import bf16_round


def blocked_unit_lower_inverse(A: np.ndarray) -> np.ndarray:
    """(I + A)^-1 for strictly lower A (64 x 64): 16 x 16 diagonal blocks by substitution, then
    off-diagonal blocks by distance from the diagonal, as the kernel's prep warps do."""
    n = A.shape[0]
    nb = n // 16
    T = np.zeros_like(A)
    for b in range(nb):
        blk = A[16 * b:16 * b + 16, 16 * b:16 * b + 16]
        for c in range(16):
            x = np.zeros(16, A.dtype)
            x[c] = 1.0
            for r in range(c + 1, 16):
                x[r] = -blk[r, c:r] @ x[c:r]
            T[16 * b:16 * b + 16, 16 * b + c] = x
    for d in range(1, nb):
        for b in range(d, nb):
            a = b - d
            X = A[16 * b:16 * b + 16, 16 * a:16 * b] @ T[16 * a:16 * b, 16 * a:16 * a + 16]
            T[16 * b:16 * b + 16, 16 * a:16 * a + 16] = -T[16 * b:16 * b + 16, 16 * b:16 * b + 16] @ X
    return T


def prefill_model(q, k, v, alpha, beta, scale, valid=None, reset=None, initial=None, C=64,
                  rounding=True):
    """Scalar-gate GDN-2 prefill exactly as the kernel computes it.  Inputs as the C ABI.
    Returns (out [B,T,H,V] f32, final_state [B,H,K,V] f32)."""
    rnd = bf16_round if rounding else (lambda x: np.asarray(x, np.float32))

    def pair(x):  # value carried as bf16 hi + bf16 lo
        x = np.asarray(x, np.float32)
        hi = rnd(x)
        return hi + rnd(x - hi)
    q, k, v = (np.asarray(x, np.float32) for x in (q, k, v))
    B, T, H, K = q.shape
    V = v.shape[3]
    out = np.zeros((B, T, H, V), np.float32)
    fin = np.zeros((B, H, K, V), np.float32)
    nch = (T + C - 1) // C
    for b in range(B):
        for h in range(H):
            S = np.zeros((K, V), np.float32) if initial is None else np.array(initial[b, h], np.float32)
            for c in range(nch):
                t0 = c * C
                n = min(C, T - t0)
                vf = np.zeros(C, np.float32)
                be = np.zeros(C, np.float32)
                a = np.ones(C, np.float32)
                for r in range(n):
                    t = t0 + r
                    ok = True if valid is None else bool(valid[b, t])
                    rs = False if reset is None else bool(reset[b, t])
                    vf[r] = 1.0 if ok else 0.0
                    if ok:
                        a[r] = 0.0 if rs else alpha[b, t, h]
                        be[r] = beta[b, t, h]
                z = (a <= 0).astype(np.int64)
                lg = np.where(z == 1, 0.0, np.log(np.where(a > 0, a, 1.0))).astype(np.float32)
                g = np.cumsum(lg, dtype=np.float32)
                cnt = np.cumsum(z)
                gamma = np.where(cnt == 0, np.exp(g), 0.0).astype(np.float32)
                same = cnt[:, None] == cnt[None, :]
                dec = np.where(same, np.exp(g[:, None] - g[None, :]), 0.0).astype(np.float32)
                Kc = np.zeros((C, K), np.float32)
                Qc = np.zeros((C, K), np.float32)
                Vc = np.zeros((C, V), np.float32)
                Kc[:n] = k[b, t0:t0 + n, h]
                Qc[:n] = q[b, t0:t0 + n, h]
                Vc[:n] = v[b, t0:t0 + n, h]
                low = np.tril(np.ones((C, C), bool), -1)
                incl = np.tril(np.ones((C, C), bool), 0)
                A = np.where(low, be[:, None] * dec * (Kc @ Kc.T), 0.0).astype(np.float32)
                P = pair(np.where(incl, scale * dec * (Qc @ Kc.T), 0.0))
                Tm = rnd(blocked_unit_lower_inverse(A))
                Sb = rnd(S)
                KS = Kc @ Sb
                QS = Qc @ Sb
                R = pair(be[:, None] * Vc - (be * gamma)[:, None] * KS)
                Delta = Tm @ R
                Dt = rnd(Delta * dec[C - 1][:, None])
                Dp = rnd(Delta)
                S = (gamma[C - 1] * S + Kc.T @ Dt).astype(np.float32)
                O = np.where(vf[:, None] != 0, (scale * gamma)[:, None] * QS + P @ Dp, 0.0)
                out[b, t0:t0 + n, h] = rnd(O[:n])
            fin[b, h] = S
    return out, fin
