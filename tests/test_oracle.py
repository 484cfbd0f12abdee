"""CPU tests of the oracle: it is pinned before anything is checked against it.

* known answers of the reference's own tests (padding preserves state and writes exact zeros,
  gdn2_reference.rs:218-235; relay single effective key / equal-key normaliser,
  relay_tests.rs:12-90);
* the reference's own cross-check: the chunkwise solver (chunk.rs) against the f64 sequential
  oracle at 2e-5 + 3e-4|ref| on its fixtures, for chunk sizes 1, 2, 5, 16 (chunk_tests.rs:171-230)
  and on the sinusoidal + edge-case fixture (checks.rs / kron_checks.rs);
* closed-form answers derived from the recurrence;
* two independent restatements (C and numpy) agreeing to rounding;
* the committed golden fixtures (tests/golden/make_golden.py) reproduced.
"""
import os

import numpy as np
import pytest

from fixtures import (chunk_test_fixture, edge_edits, edge_initial, ref_close, sinusoid_fixture,
                      splitmix_tokens)
from oracle import oracle as O

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "gdn2_golden.npz")


def test_padding_preserves_state_and_outputs_zero():
    # gdn2_reference.rs:218-235: tokens (start, end) = (0,2), (1,0) [padding], (0,2).
    K, V = 32, 64
    tok = [np.full(K, 0.1), np.full(K, 0.1), np.full(V, 0.2), np.full(K, 0.9), np.full(K, 0.3),
           np.full(V, 0.5)]
    fields = [np.broadcast_to(x, (1, 3, 1, x.size)).copy() for x in tok]
    starts = np.array([[0, 1, 0]], np.int32)
    ends = np.array([[2, 0, 2]], np.int32)
    out = O.doc_scan(*fields, starts, ends)
    assert np.all(out[0, 1] == 0.0)
    _, _, _, states = O.scan(*fields, valid=ends >= starts, reset=starts == np.arange(3),
                             return_states=True)
    assert np.array_equal(states[0, 0, 0], states[0, 0, 1])


def test_aligned_closed_form():
    # q = k = e0, v = e0, alpha = 1, erase = write = 1/2 (Fixture::aligned, checks.rs:181-198):
    # S00 <- (1 + S00) / 2, so o_t = 1 - 2^-n with n valid tokens since the last reset.
    B, T, H, K, V = 1, 12, 1, 8, 8
    e0k = np.zeros(K); e0k[0] = 1.0
    e0v = np.zeros(V); e0v[0] = 1.0
    q = np.broadcast_to(e0k, (B, T, H, K)).copy()
    v = np.broadcast_to(e0v, (B, T, H, V)).copy()
    a = np.ones((B, T, H, K))
    e = np.full((B, T, H, K), 0.5)
    w = np.full((B, T, H, V), 0.5)
    valid = np.ones((B, T), bool); valid[0, 4] = False
    reset = np.zeros((B, T), bool); reset[0, 7] = True
    out, fin, sco = O.scan(q, q, v, a, e, w, valid, reset)
    n, expect, exp_score = 0, [], []
    for t in range(T):
        if not valid[0, t]:
            expect.append(0.0); exp_score.append(0.0); continue
        if reset[0, t]:
            n = 0
        n += 1
        expect.append(1.0 - 2.0 ** -n)
        exp_score.append(2.0 ** -n)
    np.testing.assert_allclose(out[0, :, 0, 0], expect, rtol=0, atol=1e-15)
    np.testing.assert_allclose(sco[0, :, 0], exp_score, rtol=0, atol=1e-15)
    assert np.all(out[0, :, 0, 1:] == 0.0)


def test_unit_key_projection_closed_form():
    # beta = 1, alpha = 1, |k| = 1: S' = (I - k k^T) S + k v^T, so k^T S' = v exactly.
    rng = np.random.default_rng(3)
    K, V = 16, 8
    S0 = rng.standard_normal((1, 1, K, V))
    k = rng.standard_normal(K); k /= np.linalg.norm(k)
    v = rng.standard_normal(V)
    fields = [k[None, None, None], k[None, None, None], v[None, None, None],
              np.ones((1, 1, 1, K)), np.ones((1, 1, 1, K)), np.ones((1, 1, 1, V))]
    out, fin, _ = O.scan(*fields, initial=S0)
    np.testing.assert_allclose(k @ fin[0, 0], v, atol=1e-12)
    np.testing.assert_allclose(out[0, 0, 0], v, atol=1e-12)  # q = k


def test_decay_only_closed_form():
    # k = 0: no edits; o_t = (prod alpha) q^T S0.
    rng = np.random.default_rng(4)
    B, T, H, K, V = 1, 6, 1, 4, 5
    S0 = rng.standard_normal((B, H, K, V))
    q = rng.standard_normal((B, T, H, K))
    alpha = rng.uniform(0.5, 1.0, (B, T, H, K))
    z = np.zeros((B, T, H, K))
    out, fin, _ = O.scan(q, z, rng.standard_normal((B, T, H, V)), alpha, z + 0.5,
                         np.full((B, T, H, V), 0.5), initial=S0)
    decay = np.cumprod(alpha[0, :, 0], axis=0)
    for t in range(T):
        np.testing.assert_allclose(out[0, t, 0], (q[0, t, 0] * decay[t]) @ S0[0, 0], atol=1e-12)


def test_c_and_numpy_restatements_agree():
    f = splitmix_tokens(11, 2, 19, 3, 6, 7)
    rng = np.random.default_rng(0)
    valid = rng.random((2, 19)) > 0.2
    reset = rng.random((2, 19)) > 0.8
    init = rng.standard_normal((2, 3, 6, 7))
    a = O.scan(*f, valid, reset, init)
    b = O.scan_numpy(*f, valid, reset, init)
    for x, y in zip(a, b):
        np.testing.assert_allclose(x, y, rtol=0, atol=1e-12)


def test_step_matches_scan_of_one_token():
    f = splitmix_tokens(5, 3, 1, 2, 8, 8)
    init = np.random.default_rng(1).standard_normal((3, 2, 8, 8))
    out, fin, _ = O.scan(*f, initial=init)
    so, ss = O.step(*(x[:, 0].reshape(6, -1) for x in f), init.reshape(6, 8, 8))
    np.testing.assert_allclose(so.reshape(3, 1, 2, 8), out, atol=1e-13)
    np.testing.assert_allclose(ss.reshape(3, 2, 8, 8), fin, atol=1e-13)


@pytest.mark.parametrize("chunk", [1, 2, 5, 16])
def test_chunk_solver_matches_sequential_on_reference_fixture(chunk):
    # chunk_tests.rs:171-230: output at 2e-5 + 3e-4|ref| for every computational partition.
    fields, valid, reset, initial = chunk_test_fixture()
    ref_out, ref_fin, ref_sc = O.scan(*fields, valid, reset, initial)
    out, fin, sc = O.chunk_scan_f32(*fields, valid.astype(np.float32), reset.astype(np.float32),
                                    initial, chunk=chunk)
    for a, e in ((out, ref_out), (fin, ref_fin), (sc, ref_sc)):
        ok, err = ref_close(a, e)
        assert ok, err
    # padding rows output exactly zero (chunk_tests.rs:158-161)
    assert np.all(ref_out[~valid] == 0.0)


@pytest.mark.parametrize("t", [1, 7, 35])
def test_chunk_solver_matches_sequential_on_edge_fixture(t):
    # gdn_numerical_checks_selected (kron_checks.rs:89-122): T in {1, 7, 35} with the edge edits.
    fields, valid, reset = sinusoid_fixture(t)
    fields, valid, reset = edge_edits(fields, valid, reset)
    init = edge_initial()
    ref = O.scan(*fields, valid, reset, init)
    got = O.chunk_scan_f32(*fields, valid.astype(np.float32), reset.astype(np.float32), init,
                           chunk=16)
    for a, e in zip(got, ref):
        ok, err = ref_close(a, e)
        assert ok, err


def test_chunk_size_limit():
    fields, valid, reset, initial = chunk_test_fixture()
    with pytest.raises(ValueError, match="1..=16"):
        O.chunk_scan_f32(*fields, chunk=17)


def test_nonfinite_input_is_rejected():
    f = splitmix_tokens(1, 1, 2, 1, 4, 4)
    f[0][0, 1, 0, 0] = np.nan
    with pytest.raises(ValueError, match="nonfinite"):
        O.scan(*f)


def test_relay_single_effective_key_is_exact():
    # relay_tests.rs:12-45: q = 1e16, key = -1e16 (score -8e32), relays at -1.6e33 underflow to
    # zero weight: the output is exactly the one key's value, normalisation [< -1e30, 1].
    D = 64
    q = np.full((1, 1, D), 1e16, np.float32)
    ko = np.full((1, 1, 1, D), -1e16, np.float32)
    vo = (np.arange(D, dtype=np.float32) - 32.0).reshape(1, 1, 1, D)
    kp = np.full((1, 16, D), -2e16, np.float32)
    vp = np.full((1, 16, D), 23.0, np.float32)
    for fn in (O.relay_online_f32, O.relay_merge):
        o, mx, sm = fn(q, kp, vp, ko, vo, 0.125)
        assert np.isfinite(mx[0, 0]) and mx[0, 0] < -1e30
        assert sm[0, 0] == 1.0
        assert np.array_equal(np.asarray(o, np.float32)[0, 0], vo[0, 0, 0])


def test_relay_equal_keys_normaliser_is_exact():
    # relay_tests.rs:47-90: 2 + 16 identical scores give a normaliser of exactly 18.
    D = 64
    q = np.full((1, 1, D), 1e16, np.float32)
    ko = np.full((1, 1, 2, D), -1e16, np.float32)
    kp = np.full((1, 16, D), -1e16, np.float32)
    z_o = np.zeros((1, 1, 2, D), np.float32)
    z_p = np.zeros((1, 16, D), np.float32)
    for fn in (O.relay_online_f32, O.relay_merge):
        o, mx, sm = fn(q, kp, z_p, ko, z_o, 0.125)
        assert sm[0, 0] == 18.0 and mx[0, 0] < -1e30
        assert np.all(np.asarray(o) == 0.0)


def test_relay_empty_row_convention():
    D = 8
    o, mx, sm = O.relay_merge(np.ones((2, 1, D)), np.zeros((1, 0, D)), np.zeros((1, 0, D)),
                              np.zeros((2, 1, 3, D)), np.zeros((2, 1, 3, D)), 0.5,
                              own_len=np.array([0, 2]))
    assert np.all(o[0] == 0.0) and mx[0, 0] == 0.0 and sm[0, 0] == 1.0
    assert sm[1, 0] == 2.0


def test_relay_merge_equals_online_recurrence():
    rng = np.random.default_rng(7)
    N, H, D, Lp, Lo = 3, 2, 16, 9, 5
    q = rng.standard_normal((N, H, D)).astype(np.float32)
    kp, vp = (rng.standard_normal((H, Lp, D)).astype(np.float32) for _ in range(2))
    ko, vo = (rng.standard_normal((N, H, Lo, D)).astype(np.float32) for _ in range(2))
    own = np.array([5, 0, 3], np.int32)
    a = O.relay_merge(q, kp, vp, ko, vo, 0.25, own)
    b = O.relay_online_f32(q, kp, vp, ko, vo, 0.25, own)
    for x, y in zip(a, b):
        np.testing.assert_allclose(y, x, rtol=2e-5, atol=2e-6)


def test_relay_window_reference_layout():
    # relay_attention_kernel.rs:38-130 layout: window +-radius inside the document plus the
    # document's relay slots; padding rows o = 0, [0, 1].  Cross-check against relay_merge by
    # building the same key set explicitly.
    rng = np.random.default_rng(9)
    B, H, T, D, slots, radius = 1, 2, 12, 8, 3, 2
    q, k, v = (rng.standard_normal((B, H, T, D)) for _ in range(3))
    rk, rv = (rng.standard_normal((2, H, slots, D)) for _ in range(2))
    doc_id = np.array([[0] * 7 + [1] * 4 + [0]], np.int32)
    ds = np.array([[0] * 7 + [7] * 4 + [11]], np.int32)
    de = np.array([[6] * 7 + [10] * 4 + [10]], np.int32)  # last token: padding (end < start)
    o, norm = O.relay_window(q, k, v, rk, rv, doc_id, ds, de, radius=radius, scale=0.5)
    assert np.all(o[0, :, 11] == 0.0) and np.all(norm[0, :, 11] == [0.0, 1.0])
    t = 8
    keys = [j for j in range(max(0, t - radius), min(T, t + radius + 1)) if 7 <= j <= 10]
    for h in range(H):
        lo = len(keys)
        ko = k[0, h, keys][None, None]
        vo = v[0, h, keys][None, None]
        e, mx, sm = O.relay_merge(q[0, h, t][None, None], rk[1, h][None], rv[1, h][None], ko, vo, 0.5)
        np.testing.assert_allclose(o[0, h, t], e[0, 0], atol=1e-12)
        np.testing.assert_allclose(norm[0, h, t], [mx[0, 0], sm[0, 0]], atol=1e-12)


@pytest.mark.skipif(not os.path.exists(GOLDEN), reason="golden fixtures not generated")
def test_golden_fixtures_reproduce():
    import importlib.util
    spec = importlib.util.spec_from_file_location(
        "make_golden", os.path.join(os.path.dirname(__file__), "golden", "make_golden.py"))
    mg = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mg)
    stored = np.load(GOLDEN)
    fresh = mg.compute()
    assert set(stored.files) == set(fresh)
    for name in stored.files:
        np.testing.assert_allclose(fresh[name], stored[name], rtol=1e-12, atol=1e-14, err_msg=name)


def test_training_backward_matches_finite_differences():
    # The backward oracle (gdn_training.rs:117-284 restated) against central differences of the
    # forward oracle, for L = sum g_out.out + sum g_fin.final + sum g_score.scores, with padding,
    # a reset, an initial state and score gradients -- the finite-difference style of
    # gdn2_reference.rs:237-268.
    rng = np.random.default_rng(7)
    B, T, H, K, V = 1, 9, 2, 3, 4
    q, k = rng.standard_normal((B, T, H, K)), rng.standard_normal((B, T, H, K))
    v, w = rng.standard_normal((B, T, H, V)), rng.random((B, T, H, V))
    a, e = rng.uniform(0.5, 1.0, (B, T, H, K)), rng.random((B, T, H, K))
    valid = np.ones((B, T), bool)
    valid[0, 4] = False
    reset = np.zeros((B, T), bool)
    reset[0, 6] = True
    init = 0.3 * rng.standard_normal((B, H, K, V))
    go, gf, gs = rng.standard_normal((B, T, H, V)), rng.standard_normal((B, H, K, V)), rng.standard_normal((B, T, H))
    inputs = [q, k, v, a, e, w, init]

    def loss(xs):
        o, f, s = O.scan(*xs[:6], valid, reset, xs[6])
        return float(np.sum(go * o) + np.sum(gf * f) + np.sum(gs * s))
    grads = O.training_backward(q, k, v, a, e, w, go, gf, gs, valid, reset, init)
    # dq, dk, dv, dalpha, derase, dwrite, dinitial  <->  inputs q, k, v, alpha, erase, write, initial
    for gi, xi in zip(grads, [0, 1, 2, 3, 4, 5, 6]):
        x = inputs[xi]
        num = np.zeros_like(x)
        it = np.nditer(x, flags=["multi_index"])
        for _ in it:
            idx = it.multi_index
            hi = [y.copy() for y in inputs]
            lo = [y.copy() for y in inputs]
            hi[xi][idx] += 1e-6
            lo[xi][idx] -= 1e-6
            num[idx] = (loss(hi) - loss(lo)) / 2e-6
        assert np.max(np.abs(gi - num)) < 1e-6 * (1 + np.max(np.abs(num))), xi
    # padding tokens get no gradient
    for g in grads[:6]:
        assert np.all(g[0, 4] == 0.0)


@pytest.mark.parametrize("t,c,width", [(1, 3, 4), (2, 35, 4), (7, 3, 4), (17, 128, 4), (19, 256, 4), (7, 35, 1)])
def test_causal_conv_matches_reference_fixture(t, c, width):
    # The reference's convolution check (crates/mixers/src/convolution_checks.rs:55-175) restated:
    # its sin fixtures, padding/reset pattern and explicit f64 loop over lags and document masks.
    b = 2
    x = np.array([np.sin((i * 17 + 3) * 0.013) for i in range(b * t * c)], np.float32).reshape(b, t, c)
    w = np.array([0.0 if i % 7 == 0 else np.sin((i + 3) * np.float32(0.17)) * 0.1 for i in range(width * c)],
                 np.float32).reshape(width, c)
    valid = np.array([0.0 if (i % 7 == 3 or i % t == t - 1) else 1.0 for i in range(b * t)], np.float32).reshape(b, t)
    reset = np.array([1.0 if (i % t in (0, 2, 5)) else 0.0 for i in range(b * t)], np.float32).reshape(b, t)
    docs = np.cumsum(valid * reset, axis=1)
    y = np.zeros((b, t, c))
    for row in range(b):
        for dest in range(t):
            for lag in range(min(width, dest + 1)):
                src = dest - lag
                m = float(valid[row, src]) * float(valid[row, dest]) if docs[row, src] == docs[row, dest] else 0.0
                y[row, dest] += x[row, src].astype(np.float64) * w[lag].astype(np.float64) * m
    assert np.max(np.abs(O.causal_conv(x, w, valid, reset) - y)) < 1e-12


def test_prologue_gate_and_norm_known_values():
    # softplus threshold 20 (decay.rs:13-20): above it alpha = exp(-(x + b) e^s) exactly
    z = np.array([25.0, 20.5, -3.0, 0.0])
    sp = O.softplus20(z)
    assert sp[0] == 25.0 and sp[1] == 20.5
    assert abs(sp[2] - np.log1p(np.exp(-3.0))) < 1e-15 and abs(sp[3] - np.log(2.0)) < 1e-15
    # L2 rows (normalization.rs:21-25): unit norm up to eps, a zero row stays zero
    x = np.array([[3.0, 4.0], [0.0, 0.0]])
    n = O.l2_rows(x)
    assert abs(np.linalg.norm(n[0]) - 5.0 / np.sqrt(25.0 + 1e-6)) < 1e-15 and np.all(n[1] == 0.0)


def packed_layout(docs_per_row, tokens):
    """doc_id / doc_start / doc_end [B,T] of a packed batch (dre-core lib.rs:105-113, 145-175):
    documents numbered across rows, inclusive limits; a padding token has start = position,
    end = position - 1 and document id -1."""
    B = len(docs_per_row)
    di = np.full((B, tokens), -1, np.int32)
    ds = np.tile(np.arange(tokens, dtype=np.int32), (B, 1))
    de = ds - 1
    doc = 0
    for b, docs in enumerate(docs_per_row):
        first = 0
        for n in docs:
            di[b, first:first + n], ds[b, first:first + n], de[b, first:first + n] = doc, first, first + n - 1
            first += n
            doc += 1
    return di, ds, de


def test_relay_window_extreme_single_effective_key():
    # relay_tests.rs:12-47: q = 1e16, k = -1e16 (source score -8e32), relay keys -2e16 (-1.6e33):
    # every relay weight underflows, the output is exactly the one source value and the statistic
    # is (a finite maximum below -1e30, 1); the padding row gives (0, 1) and zeros.
    di, ds, de = packed_layout([[1]], 2)
    q = np.full((1, 1, 2, 64), 1e16)
    k = np.full((1, 1, 2, 64), -1e16)
    v = np.array([i - 32.0 if i < 64 else 17.0 for i in range(128)]).reshape(1, 1, 2, 64)
    rk, rv = np.full((1, 1, 16, 64), -2e16), np.full((1, 1, 16, 64), 23.0)
    o, norm = O.relay_window(q, k, v, rk, rv, di, ds, de)
    assert np.isfinite(norm[0, 0, 0, 0]) and norm[0, 0, 0, 0] < -1e30
    assert norm[0, 0, 0, 1] == 1.0
    assert list(norm[0, 0, 1]) == [0.0, 1.0]
    assert np.array_equal(o[0, 0, 0], v[0, 0, 0]) and np.all(o[0, 0, 1] == 0.0)


def test_relay_window_extreme_equal_keys():
    # relay_tests.rs:51-93: two source keys and sixteen relay keys with identical scores near -8e32:
    # the sum is exactly 18 and the output 0 for zero values.
    di, ds, de = packed_layout([[2]], 2)
    q = np.full((1, 1, 2, 64), 1e16)
    k = np.full((1, 1, 2, 64), -1e16)
    rk = np.full((1, 1, 16, 64), -1e16)
    z = np.zeros((1, 1, 2, 64))
    o, norm = O.relay_window(q, k, z, rk, np.zeros((1, 1, 16, 64)), di, ds, de)
    for row in norm[0, 0]:
        assert np.isfinite(row[0]) and row[0] < -1e30 and row[1] == 18.0
    assert np.all(o == 0.0)


def test_relay_window_matches_dense_masked_attention():
    # relay_tests.rs:94-140: tokens 6, documents [2, 3] packed; a dense softmax over
    # [window keys ; all relay slots] with the reference test's mask (other document or more than
    # 128 tokens away; relay slot of another document) equals the windowed relay attention.
    tokens, documents = 6, 2
    make = lambda n, seed: np.sin(((np.arange(n) * 31 + seed).astype(np.float32) * np.float32(0.0021))  # noqa: E731
                                  .astype(np.float32)).astype(np.float64)
    q, k, v = (make(tokens * 64, s).reshape(1, 1, tokens, 64) for s in (1, 2, 3))
    rk, rv = (make(documents * 16 * 64, s).reshape(documents, 1, 16, 64) for s in (4, 5))
    di, ds, de = packed_layout([[2, 3]], tokens)
    o, norm = O.relay_window(q, k, v, rk, rv, di, ds, de)
    docs = [0, 0, 1, 1, 1, -1]
    dk = np.concatenate([k[0, 0], rk.reshape(documents * 16, 64)])
    dv = np.concatenate([v[0, 0], rv.reshape(documents * 16, 64)])
    for t in range(tokens):
        if docs[t] < 0:
            assert np.all(o[0, 0, t] == 0.0) and list(norm[0, 0, t]) == [0.0, 1.0]
            continue
        keep = np.array([(docs[j] == docs[t] and abs(t - j) <= 128) if j < tokens else (j - tokens) // 16 == docs[t]
                         for j in range(tokens + documents * 16)])
        s = dk[keep] @ q[0, 0, t] * 0.125
        w = np.exp(s - s.max())
        np.testing.assert_allclose(o[0, 0, t], w @ dv[keep] / w.sum(), rtol=1e-12, atol=1e-14)
        np.testing.assert_allclose(norm[0, 0, t], [s.max(), w.sum()], rtol=1e-12)


def test_doc_scan_backward_matches_finite_differences():
    # gdn2_backward (gdn2.rs:285-519) restated as the stateful backward on the document masks: its
    # gradients equal central differences of the doc-limit forward oracle (gdn2_reference.rs:87-105)
    rng = np.random.default_rng(3)
    B, T, H, K, V = 1, 10, 1, 3, 4
    q, k = rng.standard_normal((B, T, H, K)), rng.standard_normal((B, T, H, K))
    v, w = rng.standard_normal((B, T, H, V)), rng.random((B, T, H, V))
    a, e = rng.uniform(0.5, 1.0, (B, T, H, K)), rng.random((B, T, H, K))
    # documents [0, 4), [4, 8), then padding at 8 and 9
    ds = np.array([[0, 0, 0, 0, 4, 4, 4, 4, 8, 9]], np.int32)
    de = np.array([[3, 3, 3, 3, 7, 7, 7, 7, 7, 8]], np.int32)
    go = rng.standard_normal((B, T, H, V))
    inputs = [q, k, v, a, e, w]

    def loss(xs):
        return float(np.sum(go * O.doc_scan(*xs, ds, de)))
    grads = O.doc_backward(q, k, v, a, e, w, ds, de, go)
    for xi, gi in enumerate(grads):
        x = inputs[xi]
        num = np.zeros_like(x)
        it = np.nditer(x, flags=["multi_index"])
        for _ in it:
            idx = it.multi_index
            hi = [y.copy() for y in inputs]
            lo = [y.copy() for y in inputs]
            hi[xi][idx] += 1e-6
            lo[xi][idx] -= 1e-6
            num[idx] = (loss(hi) - loss(lo)) / 2e-6
        assert np.max(np.abs(gi - num)) < 1e-6 * (1 + np.max(np.abs(num))), xi
