"""Input fixtures and comparison rules, restated from the reference's own tests.

The reference ships no stored vectors; its fixtures are formulas, restated here:
  * ``sinusoid_fixture``   crates/mixers/src/checks.rs:119-180 (Fixture::new)
  * ``edge_edits``         crates/mixers/src/kron_checks.rs:132-175 (check(): reset on padding,
                           an all-padding chunk, exact-zero edit, negative write, zero k / v,
                           zero decay, L2-normalised k and v)
  * ``chunk_test_fixture`` crates/mixers/src/chunk_tests.rs:25-75 (initial/reset/padding case)
  * ``SplitMix``           reuse/crates/dre-gdn2/src/tests.rs:7-33 (deterministic generator)
  * ``baseline_inputs``    BASELINE.json configs: q,k ~ N(0,1) L2-normalised per head row,
                           v ~ N(0,1), beta = sigmoid(N(0,1)), log alpha = logsigmoid(N(3,1))
Comparison rules:
  * ``ref_close``  |a - e| <= atol + rtol |e| with a hard failure on non-finite values
                   (checks.rs:73-101; ATOL 2e-5, RTOL 3e-4 for f32 against the f64 oracle)
  * ``rel_err``    max |a - e| / (|e| + rms(e)): the north-star "max relative error" with an
                   rms-scaled absolute floor, the form of the predecessor's bf16 gate
                   (reuse/crates/dre-gdn2/src/tests.rs:109-122).  Bounds: 2e-3 f32, 2e-2 bf16.
"""
from __future__ import annotations

import numpy as np

ATOL = 2e-5
RTOL = 3e-4
TOL_F32 = 2e-3
TOL_BF16 = 2e-2


def ref_close(actual, expected, atol=ATOL, rtol=RTOL):
    a = np.asarray(actual, np.float64)
    e = np.asarray(expected, np.float64)
    assert a.shape == e.shape, (a.shape, e.shape)
    if not (np.isfinite(a).all() and np.isfinite(e).all()):
        return False, float("inf")
    err = np.abs(a - e)
    return bool((err <= atol + rtol * np.abs(e)).all()), float(err.max(initial=0.0))


def rel_err(actual, expected) -> float:
    a = np.asarray(actual, np.float64)
    e = np.asarray(expected, np.float64)
    assert a.shape == e.shape, (a.shape, e.shape)
    if not np.isfinite(a).all():
        return float("inf")
    rms = float(np.sqrt(np.mean(e * e))) if e.size else 0.0
    if rms == 0.0:
        return float(np.abs(a - e).max(initial=0.0))
    return float((np.abs(a - e) / (np.abs(e) + rms)).max(initial=0.0))


def strict_metrics(actual, expected, floor=1e-3, atol=ATOL, rtol=RTOL) -> dict:
    """The three parity numbers reported beside every kernel-vs-oracle comparison:
    ``rel_err`` (above), ``max_rel`` = max |a - e| / |e| over the elements with |e| > floor * rms(e)
    (the north star's plain max relative error, with near-zero elements left out), and
    ``ref_pass`` = the fraction of elements inside the reference's |a - e| <= atol + rtol |e|
    (checks.rs:73-101, reuse/crates/dre-gdn2/src/tests.rs:109-122)."""
    a = np.asarray(actual, np.float64).ravel()
    e = np.asarray(expected, np.float64).ravel()
    assert a.shape == e.shape, (a.shape, e.shape)
    if not np.isfinite(a).all():
        return {"rel_err": float("inf"), "max_rel": float("inf"), "ref_pass": 0.0}
    rms = float(np.sqrt(np.mean(e * e))) if e.size else 0.0
    big = np.abs(e) > floor * rms
    d = np.abs(a - e)
    max_rel = float((d[big] / np.abs(e[big])).max(initial=0.0)) if big.any() else 0.0
    ref_pass = float(np.mean(d <= atol + rtol * np.abs(e))) if e.size else 1.0
    return {"rel_err": rel_err(a, e), "max_rel": max_rel, "ref_pass": ref_pass}


def report(case: str, **named) -> dict:
    """Strict metrics of each (actual, expected) pair in ``named``, printed and, when the
    environment variable DBL_PARITY_REPORT names a file, appended to it as one JSON line."""
    import json
    import os

    out = {"case": case}
    for name, (a, e) in named.items():
        out[name] = strict_metrics(a, e)
    print(json.dumps(out))
    path = os.environ.get("DBL_PARITY_REPORT")
    if path:
        with open(path, "a") as f:
            f.write(json.dumps(out) + "\n")
    return out


# ------------------------------------------------------------------------------ reference formulas
def sinusoid_fixture(t: int, b: int = 2, h: int = 4, k: int = 32, v: int = 64):
    """checks.rs:119-180 for GDN-2: returns (fields list of [B,T,H,W] f32, valid, reset)."""
    widths = [k, k, v, k, k, v]
    fields = []
    for field, width in enumerate(widths):
        i = np.arange(b * t * h * width, dtype=np.int64)
        signal = np.sin((i * 13 + field * 19 + 1).astype(np.float64) * 0.037).astype(np.float32)
        if field == 3:
            x = np.float32(0.91) + np.float32(0.03) * signal
        elif field >= 4:
            x = np.float32(0.45) + np.float32(0.1) * signal
        else:
            x = np.float32(0.1) * signal
        fields.append(x.astype(np.float32).reshape(b, t, h, width))
    idx = np.arange(b * t)
    r, p = idx // t, idx % t
    valid = ((p < np.maximum(t - (r + 1), 0)) & (p != 9) & (p != 11)).reshape(b, t)
    reset = ((p == 0) | (p == 5) | (p == 19)).reshape(b, t)
    return fields, valid, reset


def edge_edits(fields, valid, reset):
    """kron_checks.rs:132-175 edits, applied in the reference's order (in place)."""
    q, k, v, alpha, erase, write = fields
    b, t, h, _ = q.shape
    reset[0, 0] = False  # f.reset[0] = false (the flat index 0 is row 0, position 0)
    if t == 1:
        valid[:] = True
    for row in range(b):
        if t > 9:
            reset[row, 9] = True  # reset on padding must be ignored
        if row == 1 and t > 16:
            valid[row, 16:] = False  # includes an entire padding chunk
        for p in range(t):
            for hh in range(h):
                for arr in (k, v):
                    x = arr[row, p, hh]
                    norm = np.sqrt(np.sum(x * x, dtype=np.float32), dtype=np.float32)
                    arr[row, p, hh] = x / norm
                if p == 1:
                    erase[row, p, hh] = 0.0
                    write[row, p, hh] = 0.0  # exactly zero edit with nonzero key/value norms
                elif p == 3:
                    write[row, p, hh] = -0.2
                elif p == 4:
                    k[row, p, hh] = 0.0
                elif p == 6:
                    v[row, p, hh] = 0.0
                if p == 2:
                    alpha[row, p, hh, 0] = 0.0
                elif p == 16:
                    alpha[row, p, hh, :] = 0.0
    return fields, valid, reset


def edge_initial(b=2, h=4, k=32, v=64):
    """kron_checks.rs:176-178: initial_data[i] = 0.03 sin((11 i + 7) 0.017) in f32."""
    i = np.arange(b * h * k * v)
    return (np.float32(0.03) * np.sin((i * 11 + 7).astype(np.float32) * np.float32(0.017))).astype(
        np.float32).reshape(b, h, k, v)


def chunk_test_fixture():
    """chunk_tests.rs:25-75 for GDN-2: (fields, valid, reset, initial) at B2,T5,H2,K3,V4."""
    b, t, h, k, v = 2, 5, 2, 3, 4
    valid = np.array([True, False, True, True, False, True, True, False, True, False]).reshape(b, t)
    reset = np.array([False, True, False, True, False, True, False, True, False, True]).reshape(b, t)
    initial = (0.03 * (1 + np.arange(b * h * k * v) % 7)).astype(np.float32).reshape(b, h, k, v)
    widths = [k, k, v, k, k, v]
    fields = []
    for field, width in enumerate(widths):
        i = np.arange(b * t * h * width)
        if field == 3:
            x = np.where((i % (h * k) == 1) & ((i // (h * k)) % t == 2), 0.0, 0.75 + 0.02 * (i % 5))
        elif field == 4:
            x = np.full(i.shape, 0.6)
        elif field == 5:
            x = np.where((i // (h * width)) % t == 2, 0.0, -0.25)
        else:
            x = 0.08 * (((i + 3 * field) % 7) - 2.0)
        fields.append(x.astype(np.float32).reshape(b, t, h, width))
    return fields, valid, reset, initial


class SplitMix:
    """SplitMix64 (reuse/crates/dre-gdn2/src/tests.rs:7-33)."""

    MASK = (1 << 64) - 1

    def __init__(self, seed: int):
        self.state = seed & self.MASK

    def next(self) -> int:
        self.state = (self.state + 0x9E3779B97F4A7C15) & self.MASK
        z = self.state
        z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & self.MASK
        z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & self.MASK
        return z ^ (z >> 31)

    def uniform(self) -> float:
        return (self.next() >> 11) / float(1 << 53)

    def signed(self) -> float:
        return 2.0 * self.uniform() - 1.0


def splitmix_tokens(seed: int, b: int, t: int, h: int, k: int, v: int):
    """fixture_token (tests.rs:43-51) drawn for every (b, t, h): q, k, v, alpha, erase, write."""
    rng = SplitMix(seed)
    spec = [(k, 0.0, 0.5), (k, 0.0, 0.45), (v, 0.0, 1.0), (k, 0.875, 0.075), (k, 0.5, 0.2),
            (v, 0.75, 0.25)]
    out = [np.zeros((b, t, h, w), np.float64) for w, _, _ in spec]
    for bb in range(b):
        for tt in range(t):
            for hh in range(h):
                for f, (w, c, s) in enumerate(spec):
                    out[f][bb, tt, hh] = [c + s * rng.signed() for _ in range(w)]
    return out


# ------------------------------------------------------------------------------ BASELINE inputs
def baseline_inputs(seed: int, b: int, t: int, h: int, dk: int, dv: int):
    """Seeded synthetic inputs with the BASELINE value distributions (numpy default_rng)."""
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((b, t, h, dk), dtype=np.float32)
    k = rng.standard_normal((b, t, h, dk), dtype=np.float32)
    q /= np.linalg.norm(q, axis=-1, keepdims=True)
    k /= np.linalg.norm(k, axis=-1, keepdims=True)
    v = rng.standard_normal((b, t, h, dv), dtype=np.float32)
    beta = (1.0 / (1.0 + np.exp(-rng.standard_normal((b, t, h))))).astype(np.float32)
    x = rng.normal(3.0, 1.0, (b, t, h))
    alpha = np.exp(-np.logaddexp(0.0, -x)).astype(np.float32)  # exp(logsigmoid(x))
    return q, k, v, alpha, beta


def bf16_round(x) -> np.ndarray:
    """Round an f32 array to bf16 (round-to-nearest-even) and return it as f32."""
    a = np.ascontiguousarray(x, np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    return r.astype(np.uint32).view(np.float32).reshape(a.shape)
