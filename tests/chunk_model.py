"""numpy model of the tensor-core prefill kernel's arithmetic (prefill_tc.cu), for CPU tests.

It follows the kernel step by step -- log-space decay products with reset counting, the inverse
of (I + A) by block doubling, and rounding exactly where the kernel rounds an MMA operand: every
operand of the state chain is fp16 (the chunk's K and Q tiles are converted in place, Q rows
scaled by the output multiplier scale * gamma_r; S, R, T, Delta, the Gamma-scaled Delta and P),
only [K;Q] K^T runs on the bf16 input tiles -- so the numerical error budget of the kernel can be
checked against the oracle without a GPU.  Test infrastructure only.
"""
from __future__ import annotations

import numpy as np

from fixtures import bf16_round


def blocked_unit_lower_inverse(A: np.ndarray) -> np.ndarray:
    """(I + A)^-1 for strictly lower A (64 x 64) as the kernel's prep warps compute it: the 8 x 8
    diagonal blocks by substitution, then pairs of inverted n x n diagonal blocks joined into 2n x 2n
    ones (n = 8, 16, 32) through the lower-left block T10 = -T11 (A10 T00)."""
    n = A.shape[0]
    T = np.zeros_like(A)
    for b in range(n // 8):
        blk = A[8 * b:8 * b + 8, 8 * b:8 * b + 8]
        for c in range(8):
            x = np.zeros(8, A.dtype)
            x[c] = 1.0
            for r in range(c + 1, 8):
                x[r] = -blk[r, c:r] @ x[c:r]
            T[8 * b:8 * b + 8, 8 * b + c] = x
    m = 8
    while m < n:
        for a0 in range(0, n, 2 * m):
            X = A[a0 + m:a0 + 2 * m, a0:a0 + m] @ T[a0:a0 + m, a0:a0 + m]
            T[a0 + m:a0 + 2 * m, a0:a0 + m] = -T[a0 + m:a0 + 2 * m, a0 + m:a0 + 2 * m] @ X
        m *= 2
    return T


def prefill_model(q, k, v, alpha, beta, scale, valid=None, reset=None, initial=None, C=64,
                  rounding=True):
    """Scalar-gate GDN-2 prefill exactly as the kernel computes it.  Inputs as the C ABI.
    Returns (out [B,T,H,V] f32, final_state [B,H,K,V] f32)."""
    rnd = bf16_round if rounding else (lambda x: np.asarray(x, np.float32))

    def h16(x):  # fp16 MMA operand
        x = np.asarray(x, np.float32)
        return x.astype(np.float16).astype(np.float32) if rounding else x
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
                P = h16(np.where(incl, scale * dec * (Qc @ Kc.T), 0.0))
                Tm = h16(blocked_unit_lower_inverse(A))
                P = np.where(vf[:, None] != 0, P, 0.0)            # padding rows of P are zero
                Kh = h16(Kc)                                         # the K tile in fp16
                Qh = h16((vf * scale * gamma)[:, None] * Qc)         # Q rows scaled by om_r, fp16
                Sb = h16(S)
                KS = Kh @ Sb
                R = h16(be[:, None] * Vc - (be * gamma)[:, None] * KS)
                Delta = Tm @ R
                Dt = h16(Delta * dec[C - 1][:, None])
                Dp = h16(Delta)
                S = (gamma[C - 1] * S + Kh.T @ Dt).astype(np.float32)
                O = Qh @ Sb + P @ Dp
                out[b, t0:t0 + n, h] = rnd(O[:n])
            fin[b, h] = S
    return out, fin
