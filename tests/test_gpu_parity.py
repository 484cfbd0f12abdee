"""GPU parity: every kernel against the CPU oracle on the same seeded inputs.

Tolerances: f32 paths at the reference's 2e-5 + 3e-4|ref| (checks.rs:73-74) where the reference
checks f32 against f64, and the north-star bounds elsewhere (``rel_err``: 2e-3 for f32, 2e-2 for
bf16 inputs; inputs are rounded to bf16 before the oracle runs, so only kernel rounding counts).
"""
import ctypes
import os

import numpy as np
import pytest
import torch

import delta_block_lm_b200 as dbl
from delta_block_lm_b200 import _native as N
from fixtures import (TOL_BF16, TOL_F32, baseline_inputs, bf16_round, chunk_test_fixture, edge_edits,
                      edge_initial, ref_close, rel_err, sinusoid_fixture, splitmix_tokens)
from oracle import oracle as O

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "gdn2_golden.npz")


def dev_t(x, device, dtype=torch.float32):
    return torch.as_tensor(np.ascontiguousarray(x), dtype=torch.float32).to(device=device, dtype=dtype)


def host(t):
    return t.detach().float().cpu().numpy()


# ----------------------------------------------------------------------- reference contract
@pytest.mark.parametrize("t", [1, 7, 35])
def test_training_scan_matches_golden_edge_fixture(cuda, native_lib, t):
    fields, valid, reset = sinusoid_fixture(t)
    fields, valid, reset = edge_edits(fields, valid, reset)
    init = edge_initial()
    g = np.load(GOLDEN)
    args = [dev_t(x, cuda) for x in fields] + [dev_t(valid, cuda), dev_t(reset, cuda), dev_t(init, cuda)]
    r = dbl.gdn_training_scan(*args, chunk_size=16)
    torch.cuda.synchronize()
    for got, name in ((r.output, "out"), (r.final_state, "final"), (r.scores[..., 0], "scores")):
        ok, err = ref_close(host(got), g[f"edge_t{t}_{name}"])
        assert ok, (name, err)


def test_training_scan_chunk_fixture_and_padding_zero(cuda, native_lib):
    fields, valid, reset, initial = chunk_test_fixture()
    g = np.load(GOLDEN)
    r = dbl.gdn_training_scan(*[dev_t(x, cuda) for x in fields], dev_t(valid, cuda), dev_t(reset, cuda),
                              dev_t(initial, cuda), 1)
    out = host(r.output)
    ok, err = ref_close(out, g["chunk_out"])
    assert ok, err
    assert np.all(out[~valid] == 0.0)
    ok, err = ref_close(host(r.final_state), g["chunk_final"])
    assert ok, err


@pytest.mark.parametrize("K,V", [(48, 200), (100, 96), (7, 9)])
def test_training_scan_lane_layouts(cuda, native_lib, K, V):
    # widths that take each lane layout of the sequential kernel (two lanes per column above 128
    # columns, four below; rows not a multiple of the lane count), with padding, a reset and an
    # initial state, against the f64 oracle
    f = splitmix_tokens(91 + K, 2, 33, 2, K, V)
    q, k, v = (x.astype(np.float32) for x in f[:3])
    valid = np.ones((2, 33), bool)
    valid[1, 25:] = False
    reset = np.zeros((2, 33), bool)
    reset[0, 11] = True
    init = (0.1 * np.random.default_rng(K).standard_normal((2, 2, K, V))).astype(np.float32)
    out, fin, sco = O.scan(q, k, v, *f[3:], valid, reset, init)
    r = dbl.gdn_training_scan(*(dev_t(x, cuda) for x in (q, k, v, *f[3:], valid, reset, init)), 16)
    assert rel_err(host(r.output), out) < TOL_F32
    assert rel_err(host(r.final_state), fin) < TOL_F32
    assert rel_err(host(r.scores[..., 0]), sco) < TOL_F32


def test_training_scan_bf16_inputs(cuda, native_lib):
    f = splitmix_tokens(77, 2, 40, 3, 32, 64)
    q, k, v = (bf16_round(x.astype(np.float32)) for x in f[:3])
    valid = np.ones((2, 40), bool)
    valid[1, 30:] = False
    reset = np.zeros((2, 40), bool)
    reset[0, 17] = True
    init = np.zeros((2, 3, 32, 64), np.float32)
    out, fin, sco = O.scan(q, k, v, *f[3:], valid, reset, init)
    r = dbl.gdn_training_scan(dev_t(q, cuda, torch.bfloat16), dev_t(k, cuda, torch.bfloat16),
                              dev_t(v, cuda, torch.bfloat16), *[dev_t(x, cuda) for x in f[3:]],
                              dev_t(valid, cuda), dev_t(reset, cuda), dev_t(init, cuda), 16)
    assert rel_err(host(r.output), out) < TOL_F32
    assert rel_err(host(r.final_state), fin) < TOL_F32
    assert rel_err(host(r.scores[..., 0]), sco) < TOL_F32


@pytest.mark.parametrize("B,T,H,K,V", [(2, 200, 3, 64, 128), (4, 70, 16, 32, 128), (1, 97, 2, 7, 9),
                                       (3, 64, 2, 20, 36), (2, 61, 2, 37, 50), (8, 48, 16, 32, 64),
                                       (32, 48, 16, 32, 64)])
def test_training_scan_chunked_form(cuda, native_lib, B, T, H, K, V):
    # sequences of two or more 16-token chunks with key width <= 64, value width <= 128 and
    # B*H*ceil(K/32)*ceil(V/64) <= 384 take the chunked form: 16-column groups with partial score
    # sums, 32-column groups, one group (V <= 16), widths that are not multiples of 4 (4-byte staging),
    # 128 sequence-heads (256 CTAs, two per SM) and a ragged last chunk; padding runs, resets (one on
    # padding) and an initial state.  512 sequence-heads take the token-sequential kernel
    f = splitmix_tokens(300 + T + K, B, T, H, K, V)
    f[1] = f[1] / np.linalg.norm(f[1], axis=-1, keepdims=True)
    q, k, v = (x.astype(np.float32) for x in f[:3])
    rng = np.random.default_rng(T + K)
    valid = rng.random((B, T)) > 0.1
    valid[0, 40:60] = False
    reset = rng.random((B, T)) > 0.93
    reset[0, 45] = True
    init = (0.1 * rng.standard_normal((B, H, K, V))).astype(np.float32)
    out, fin, sco = O.scan(q, k, v, *f[3:], valid, reset, init)
    r = dbl.gdn_training_scan(*(dev_t(x, cuda) for x in (q, k, v, *f[3:], valid, reset, init)), 16)
    ok, err = ref_close(host(r.output), out)
    assert ok, ("out", err)
    ok, err = ref_close(host(r.final_state), fin)
    assert ok, ("final", err)
    ok, err = ref_close(host(r.scores[..., 0]), sco)
    assert ok, ("scores", err)
    assert np.all(host(r.output)[~valid] == 0.0)


def test_gdn2_scan_chunked_bf16_documents(cuda, native_lib):
    # bf16 in and out through the document-limit entry on the chunked form: documents that start
    # and end inside chunks, a padding gap and one-token documents
    B, T, H, K, V = 2, 150, 3, 32, 64
    f = splitmix_tokens(4242, B, T, H, K, V)
    f[1] = f[1] / np.linalg.norm(f[1], axis=-1, keepdims=True)
    f[:3] = [bf16_round(x.astype(np.float32)) for x in f[:3]]
    bounds = [0, 23, 24, 61, 90, 131, 150]
    starts = np.zeros((B, T), np.int32)
    ends = np.zeros((B, T), np.int32)
    for lo, hi in zip(bounds[:-1], bounds[1:]):
        starts[:, lo:hi] = lo
        ends[:, lo:hi] = hi - 1
    starts[1, 70:80], ends[1, 70:80] = 80, 79  # padding: end < start
    ref = O.doc_scan(*f, starts, ends)
    out = dbl.gdn2_scan(*[dev_t(x, cuda, torch.bfloat16 if i < 3 else torch.float32) for i, x in enumerate(f)],
                        torch.as_tensor(starts, device=cuda), torch.as_tensor(ends, device=cuda))
    got = host(out)
    assert out.dtype == torch.bfloat16
    assert rel_err(got, ref) < TOL_BF16
    assert np.all(got[1, 70:80] == 0.0)


def test_gdn2_scan_doc_limits(cuda, native_lib):
    g = np.load(GOLDEN)
    f = splitmix_tokens(2024, 1, 33, 2, 32, 64)
    starts = np.array([[0] * 20 + [20] * 10 + [30, 31, 32]], np.int32)
    ends = np.array([[19] * 20 + [29] * 10 + [29, 32, 32]], np.int32)
    out = dbl.gdn2_scan(*[dev_t(x, cuda) for x in f], torch.as_tensor(starts, device=cuda),
                        torch.as_tensor(ends, device=cuda))
    got = host(out)
    ok, err = ref_close(got, g["doc_out"])
    assert ok, err
    assert np.all(got[0, 30] == 0.0)


# ----------------------------------------------------------------------- scalar-gate prefill
def _prefill_case(cuda, seed, B, T, H, Dk, Dv, dtype, initial=False, masks=False):
    q, k, v, alpha, beta = baseline_inputs(seed, B, T, H, Dk, Dv)
    if dtype == torch.bfloat16:
        q, k, v = bf16_round(q), bf16_round(k), bf16_round(v)
    rng = np.random.default_rng(seed + 100)
    init = (0.02 * rng.standard_normal((B, H, Dk, Dv))).astype(np.float32) if initial else None
    valid = reset = None
    if masks:
        valid = rng.random((B, T)) > 0.1
        reset = rng.random((B, T)) > 0.97
    ref_out, ref_fin, _ = O.scan_scalar(q, k, v, alpha, beta, valid, reset, init)
    out, fin = dbl.gdn2_prefill(dev_t(q, cuda, dtype), dev_t(k, cuda, dtype), dev_t(v, cuda, dtype),
                                dev_t(alpha, cuda), dev_t(beta, cuda),
                                valid=None if valid is None else dev_t(valid, cuda),
                                reset=None if reset is None else dev_t(reset, cuda),
                                initial_state=None if init is None else dev_t(init, cuda))
    return host(out), host(fin), ref_out, ref_fin


def test_prefill_config0_f32(cuda, native_lib):
    # BASELINE config 0 at full size: B2 H4 T512 d64 f32.
    out, fin, ro, rf = _prefill_case(cuda, 0, 2, 512, 4, 64, 64, torch.float32)
    assert rel_err(out, ro) < TOL_F32
    assert rel_err(fin, rf) < TOL_F32


@pytest.mark.parametrize("masks,initial", [(False, False), (True, True)])
def test_prefill_bf16_d128(cuda, native_lib, masks, initial):
    out, fin, ro, rf = _prefill_case(cuda, 1, 2, 200, 3, 128, 128, torch.bfloat16, initial, masks)
    assert rel_err(out, ro) < TOL_BF16
    assert rel_err(fin, rf) < TOL_BF16


def test_span_transition_composes(cuda, native_lib):
    # S_end = A S0 + B, with B the scan from zero: checked against the scan from S0.
    B, T, H, D = 1, 130, 2, 64
    q, k, v, alpha, beta = baseline_inputs(5, B, T, H, D, D)
    rng = np.random.default_rng(6)
    S0 = rng.standard_normal((B, H, D, D)).astype(np.float32) * 0.1
    _, ref_fin, _ = O.scan_scalar(q, k, v, alpha, beta, initial=S0)
    A = host(dbl.gdn2_span_transition(dev_t(k, cuda), dev_t(alpha, cuda), dev_t(beta, cuda)))
    _, Bs = dbl.gdn2_prefill(dev_t(q, cuda), dev_t(k, cuda), dev_t(v, cuda), dev_t(alpha, cuda),
                             dev_t(beta, cuda), want_output=False)
    comp = np.einsum("bhik,bhkj->bhij", A, S0) + host(Bs)
    assert rel_err(comp, ref_fin) < TOL_F32


# ----------------------------------------------------------------------- decode step
@pytest.mark.parametrize("dtype,Dk,Dv", [(torch.bfloat16, 128, 128), (torch.float32, 128, 128),
                                         (torch.bfloat16, 64, 128), (torch.float32, 64, 64)])
def test_decode_step_64_steps(cuda, native_lib, dtype, Dk, Dv):
    Nn, H, steps = 8, 4, 64
    rng = np.random.default_rng(12)
    S = (0.02 * rng.standard_normal((Nn, H, Dk, Dv))).astype(np.float32)
    state = dev_t(S, cuda)
    Sref = S.reshape(Nn * H, Dk, Dv).astype(np.float64)
    scale = 1.0 / np.sqrt(Dk)
    worst = 0.0
    for s in range(steps):
        q, k, v, alpha, beta = baseline_inputs(1000 + s, Nn, 1, H, Dk, Dv)
        q, k, v, alpha, beta = q[:, 0], k[:, 0], v[:, 0], alpha[:, 0], beta[:, 0]
        if dtype == torch.bfloat16:
            q, k, v = bf16_round(q), bf16_round(k), bf16_round(v)
        out = dbl.gdn2_decode_step(dev_t(q, cuda, dtype), dev_t(k, cuda, dtype), dev_t(v, cuda, dtype),
                                   dev_t(alpha, cuda), dev_t(beta, cuda), state)
        a = np.broadcast_to(alpha.reshape(-1, 1), (Nn * H, Dk))
        e = np.broadcast_to(beta.reshape(-1, 1), (Nn * H, Dk))
        w = np.broadcast_to(beta.reshape(-1, 1), (Nn * H, Dv))
        ro, Sref = O.step(q.reshape(-1, Dk) * scale, k.reshape(-1, Dk), v.reshape(-1, Dv), a, e, w, Sref)
        worst = max(worst, rel_err(host(out).reshape(-1, Dv), ro))
    tol = TOL_BF16 if dtype == torch.bfloat16 else TOL_F32
    assert worst < tol
    assert rel_err(host(state).reshape(-1, Dk, Dv), Sref) < tol


# ----------------------------------------------------------------------- relay merge
def _relay_case(cuda, dtype, N_, H, D, Lp, Lo, own_len=None, seed=0):
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((N_, H, D)).astype(np.float32)
    kp, vp = (rng.standard_normal((H, Lp, D)).astype(np.float32) for _ in range(2))
    ko, vo = (rng.standard_normal((N_, H, Lo, D)).astype(np.float32) for _ in range(2))
    if dtype == torch.bfloat16:
        q, kp, vp, ko, vo = (bf16_round(x) for x in (q, kp, vp, ko, vo))
    scale = 1.0 / np.sqrt(D)
    ro, rm, rs = O.relay_merge(q, kp, vp, ko, vo, scale, own_len)
    ol = None if own_len is None else torch.as_tensor(own_len, device=cuda)
    o, m, s = dbl.relay_merge_decode(dev_t(q, cuda, dtype), dev_t(kp, cuda, dtype), dev_t(vp, cuda, dtype),
                                     dev_t(ko, cuda, dtype), dev_t(vo, cuda, dtype), own_len=ol)
    return (host(o), host(m), host(s)), (ro, rm, rs)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("D", [128, 64])
def test_relay_merge_matches_oracle(cuda, native_lib, dtype, D):
    got, ref = _relay_case(cuda, dtype, 8, 4, D, 700, 300, seed=D)
    tol = TOL_BF16 if dtype == torch.bfloat16 else TOL_F32
    assert rel_err(got[0], ref[0]) < tol
    # the statistics: max is a plain score, sum = sum exp(score - max)
    assert rel_err(got[1], ref[1]) < tol and rel_err(got[2], ref[2]) < tol


def test_relay_merge_ragged_and_empty(cuda, native_lib):
    own = np.array([0, 1, 255, 256, 257, 1000, 3, 0], np.int32)
    got, ref = _relay_case(cuda, torch.bfloat16, 8, 2, 128, 64, 1000, own_len=own, seed=3)
    assert rel_err(got[0], ref[0]) < TOL_BF16
    # no prefix and no own keys: o = 0, [0, 1]
    got, ref = _relay_case(cuda, torch.bfloat16, 3, 2, 128, 0, 16, own_len=np.array([0, 4, 0], np.int32))
    assert np.all(got[0][0] == 0.0) and np.all(got[1][0] == 0.0) and np.all(got[2][0] == 1.0)
    assert rel_err(got[0][1], ref[0][1]) < TOL_BF16


@pytest.mark.parametrize("dtype,D", [(torch.bfloat16, 128), (torch.bfloat16, 64), (torch.float32, 64)])
def test_relay_merge_many_sequences_and_blocks(cuda, native_lib, dtype, D):
    # 150 sequences: three 64-query passes through every prefix block (its tile buffers and the
    # pair-exchange buffers reused across passes); a 2500-key prefix: three prefix blocks, the last
    # one short, ending in a 4-key tile; 1500 own keys: two own blocks, the second ending inside a
    # ring stage; ragged own lengths on and around the block and stage boundaries
    N_, H = 150, 2
    own = np.random.default_rng(5).integers(0, 1501, N_).astype(np.int32)
    own[:8] = [0, 1, 63, 64, 1023, 1024, 1025, 1500]
    got, ref = _relay_case(cuda, dtype, N_, H, D, 2500, 1500, own_len=own, seed=11)
    tol = TOL_BF16 if dtype == torch.bfloat16 else TOL_F32
    assert rel_err(got[0], ref[0]) < tol
    assert rel_err(got[1], ref[1]) < tol and rel_err(got[2], ref[2]) < tol
    assert native_device_ok()


def test_relay_merge_known_answers(cuda, native_lib):
    # relay_tests.rs:12-90 restated for the split layout (see tests/test_oracle.py).
    D = 64
    for dtype in (torch.float32, torch.bfloat16):
        q = torch.full((1, 1, D), 1e16, device=cuda, dtype=dtype)
        ko = torch.full((1, 1, 1, D), -1e16, device=cuda, dtype=dtype)
        vo = (torch.arange(D, device=cuda, dtype=torch.float32) - 32.0).reshape(1, 1, 1, D).to(dtype)
        kp = torch.full((1, 16, D), -2e16, device=cuda, dtype=dtype)
        vp = torch.full((1, 16, D), 23.0, device=cuda, dtype=dtype)
        o, m, s = dbl.relay_merge_decode(q, kp, vp, ko, vo, scale=0.125)
        assert torch.equal(o[0, 0].float(), vo[0, 0, 0].float())
        assert s.item() == 1.0 and m.item() < -1e30
        ko2 = torch.full((1, 1, 2, D), -1e16, device=cuda, dtype=dtype)
        kp2 = torch.full((1, 16, D), -1e16, device=cuda, dtype=dtype)
        o, m, s = dbl.relay_merge_decode(q, kp2, torch.zeros_like(kp2), ko2, torch.zeros_like(ko2), scale=0.125)
        assert s.item() == 18.0 and torch.all(o == 0)


def test_relay_workspace_is_reusable(cuda, native_lib):
    rng = np.random.default_rng(1)
    N_, H, D, Lp, Lo = 4, 2, 128, 128, 256
    ws = torch.empty(dbl.relay_workspace_bytes(N_, H, D, Lp, Lo), device=cuda, dtype=torch.uint8)
    for it in range(3):
        q = torch.randn(N_, H, D, device=cuda, dtype=torch.bfloat16)
        kp, vp = (torch.randn(H, Lp, D, device=cuda, dtype=torch.bfloat16) for _ in range(2))
        ko, vo = (torch.randn(N_, H, Lo, D, device=cuda, dtype=torch.bfloat16) for _ in range(2))
        o, _, _ = dbl.relay_merge_decode(q, kp, vp, ko, vo, workspace=ws)
        ro, _, _ = O.relay_merge(host(q), host(kp), host(vp), host(ko), host(vo), 1.0 / np.sqrt(D))
        assert rel_err(host(o), ro) < TOL_BF16


# ----------------------------------------------------------------------- tensor-core prefill
def _device_error_clear(native_lib):
    import ctypes
    code = ctypes.c_int(0)
    rc = native_lib.dbl_device_error(ctypes.byref(code))
    return rc, code.value


def test_prefill_tc_matches_model_and_oracle(cuda, native_lib):
    from chunk_model import prefill_model
    B, T, H, D = 2, 333, 2, 128  # partial last chunk
    q, k, v, alpha, beta = baseline_inputs(11, B, T, H, D, D)
    q, k, v = bf16_round(q), bf16_round(k), bf16_round(v)
    rng = np.random.default_rng(4)
    init = (0.02 * rng.standard_normal((B, H, D, D))).astype(np.float32)
    valid = rng.random((B, T)) > 0.05
    reset = rng.random((B, T)) > 0.98
    out, fin = dbl.gdn2_prefill(dev_t(q, cuda, torch.bfloat16), dev_t(k, cuda, torch.bfloat16),
                                dev_t(v, cuda, torch.bfloat16), dev_t(alpha, cuda), dev_t(beta, cuda),
                                valid=dev_t(valid, cuda), reset=dev_t(reset, cuda), initial_state=dev_t(init, cuda))
    torch.cuda.synchronize()
    assert _device_error_clear(native_lib) == (0, 0)
    out, fin = host(out), host(fin)
    ro, rf, _ = O.scan_scalar(q, k, v, alpha, beta, valid, reset, init)
    mo, mf = prefill_model(q, k, v, alpha, beta, 1 / np.sqrt(D), valid, reset, init)
    assert rel_err(out, ro) < TOL_BF16 and rel_err(fin, rf) < TOL_BF16
    assert rel_err(out, mo) < 1e-2 and rel_err(fin, mf) < 1e-2
    assert np.all(out[~valid] == 0.0)


def test_prefill_tc_config1_full_size_sampled_heads(cuda, native_lib):
    # BASELINE config 1 at full size on the GPU; two (b, h) heads checked against the oracle.
    import bench
    q, k, v, alpha, beta = bench.make_prefill_inputs(torch, cuda, 1234)
    out, fin = dbl.gdn2_prefill(q, k, v, alpha, beta)
    torch.cuda.synchronize()
    assert _device_error_clear(native_lib) == (0, 0)
    for b, h in ((0, 0), (7, 13)):
        sl = lambda t: host(t[b:b + 1, :, h:h + 1])  # noqa: E731
        ro, rf, _ = O.scan_scalar(sl(q), sl(k), sl(v), host(alpha[b:b + 1, :, h:h + 1]),
                                  host(beta[b:b + 1, :, h:h + 1]))
        assert rel_err(host(out[b:b + 1, :, h:h + 1]), ro) < TOL_BF16
        assert rel_err(host(fin[b:b + 1, h:h + 1]), rf) < TOL_BF16


def test_prefill_tc_span_transition(cuda, native_lib):
    B, T, H, D = 1, 300, 2, 128
    q, k, v, alpha, beta = baseline_inputs(21, B, T, H, D, D)
    q, k, v = bf16_round(q), bf16_round(k), bf16_round(v)
    S0 = (0.05 * np.random.default_rng(2).standard_normal((B, H, D, D))).astype(np.float32)
    _, ref_fin, _ = O.scan_scalar(q, k, v, alpha, beta, initial=S0)
    A = host(dbl.gdn2_span_transition(dev_t(k, cuda, torch.bfloat16), dev_t(alpha, cuda), dev_t(beta, cuda)))
    _, Bs = dbl.gdn2_prefill(dev_t(q, cuda, torch.bfloat16), dev_t(k, cuda, torch.bfloat16),
                             dev_t(v, cuda, torch.bfloat16), dev_t(alpha, cuda), dev_t(beta, cuda),
                             want_output=False)
    torch.cuda.synchronize()
    assert _device_error_clear(native_lib) == (0, 0)
    comp = np.einsum("bhik,bhkj->bhij", A, S0) + host(Bs)
    assert rel_err(comp, ref_fin) < TOL_BF16


# ----------------------------------------------------------------------- training-scan backward
@pytest.mark.parametrize("K,V,chunk", [(32, 64, 16), (64, 128, 5), (20, 40, 1), (48, 160, 7), (24, 200, 16)])
def test_training_backward_matches_oracle(cuda, native_lib, K, V, chunk):
    # gdn_training_backward (gdn_training.rs:117-284) against the f64 oracle, which is itself
    # pinned by finite differences (tests/test_oracle.py); padding, resets, an initial state and
    # all three upstream gradients.
    rng = np.random.default_rng(K + V)
    B, T, H = 2, 37, 3
    q, k = rng.standard_normal((B, T, H, K)) / np.sqrt(K), rng.standard_normal((B, T, H, K)) / np.sqrt(K)
    v, w = rng.standard_normal((B, T, H, V)), rng.random((B, T, H, V))
    a, e = rng.uniform(0.6, 1.0, (B, T, H, K)), rng.random((B, T, H, K))
    valid = rng.random((B, T)) > 0.1
    reset = rng.random((B, T)) > 0.93
    init = 0.1 * rng.standard_normal((B, H, K, V))
    go, gf, gs = rng.standard_normal((B, T, H, V)), rng.standard_normal((B, H, K, V)), rng.standard_normal((B, T, H))
    d = lambda x: torch.as_tensor(np.asarray(x, np.float32), device=cuda)  # noqa: E731
    got = dbl.gdn_training_backward(d(q), d(k), d(v), d(a), d(e), d(w), d(valid), d(reset), d(init), d(go),
                                    d(gf), d(gs), chunk_size=chunk)
    torch.cuda.synchronize()
    ref = O.training_backward(*(np.asarray(x, np.float32) for x in (q, k, v, a, e, w, go, gf, gs)), valid, reset,
                              np.asarray(init, np.float32))
    names = ("dq", "dk", "dv", "dalpha", "derase", "dwrite", "dinitial")
    for name, r in zip(names, ref):
        g = getattr(got, name).cpu().numpy()
        assert rel_err(g, r) < TOL_F32, (name, rel_err(g, r))
    for name in names[:6]:
        assert np.all(getattr(got, name).cpu().numpy()[~valid] == 0.0), name


@pytest.mark.parametrize("B,T,H,K,V,opt", [(2, 70, 3, 32, 64, True), (1, 50, 2, 64, 128, True),
                                           (2, 37, 2, 7, 9, True), (3, 64, 2, 20, 36, False),
                                           (2, 45, 2, 37, 50, True), (4, 96, 16, 32, 64, True),
                                           (8, 40, 16, 32, 64, True)])
def test_training_backward_chunked_form(cuda, native_lib, B, T, H, K, V, opt):
    # 16-token checkpoints with key width <= 64, value width <= 128 and T >= 32 take the chunked
    # backward (128 sequence-heads here, 256 CTAs of the reverse pass): ragged last
    # chunks, widths that are not multiples of 4, padding runs,
    # resets (one on padding), a zero gate in one channel, and with / without an initial state and
    # the final-state and score gradients, against the f64 oracle
    rng = np.random.default_rng(K * 7 + T)
    q, k = rng.standard_normal((B, T, H, K)) / np.sqrt(K), rng.standard_normal((B, T, H, K)) / np.sqrt(K)
    v, w = rng.standard_normal((B, T, H, V)), rng.random((B, T, H, V))
    a, e = rng.uniform(0.6, 1.0, (B, T, H, K)), rng.random((B, T, H, K))
    a[0, 5, 0, 1] = 0.0
    valid = rng.random((B, T)) > 0.1
    valid[0, 20:34] = False
    reset = rng.random((B, T)) > 0.93
    reset[0, 25] = True
    init = 0.1 * rng.standard_normal((B, H, K, V)) if opt else np.zeros((B, H, K, V))
    go = rng.standard_normal((B, T, H, V))
    gf = rng.standard_normal((B, H, K, V)) if opt else np.zeros((B, H, K, V))
    gs = rng.standard_normal((B, T, H)) if opt else np.zeros((B, T, H))
    d = lambda x: torch.as_tensor(np.asarray(x, np.float32), device=cuda)  # noqa: E731
    got = dbl.gdn_training_backward(d(q), d(k), d(v), d(a), d(e), d(w), d(valid), d(reset), d(init), d(go),
                                    d(gf) if opt else None, d(gs) if opt else None, chunk_size=16)
    torch.cuda.synchronize()
    ref = O.training_backward(*(np.asarray(x, np.float32) for x in (q, k, v, a, e, w, go, gf, gs)), valid, reset,
                              np.asarray(init, np.float32))
    names = ("dq", "dk", "dv", "dalpha", "derase", "dwrite", "dinitial")
    for name, r in zip(names, ref):
        g = getattr(got, name).cpu().numpy()
        assert rel_err(g, r) < TOL_F32, (name, rel_err(g, r))
    for name in names[:6]:
        assert np.all(getattr(got, name).cpu().numpy()[~valid] == 0.0), name


@pytest.mark.parametrize("B,T,H,K,V,chunk", [(2, 70, 3, 32, 64, 16), (8, 40, 16, 32, 64, 16), (1, 50, 2, 64, 128, 16),
                                             (2, 37, 2, 32, 64, 8)])
def test_training_saved_context(cuda, native_lib, B, T, H, K, V, chunk):
    # the forward -> backward hand-off (the reference's checkpoint and auxiliary tensors): the saved
    # forward gives the plain forward's outputs, and the backward from its context gives exactly the
    # recomputing backward's gradients (the same kernels on the same maps), within the f32 bound of
    # the f64 oracle; 128 sequence-heads (beyond the plain forward's chunked form) and a shape with
    # no context (chunk 8)
    rng = np.random.default_rng(K + T + chunk)
    q, k = rng.standard_normal((B, T, H, K)) / np.sqrt(K), rng.standard_normal((B, T, H, K)) / np.sqrt(K)
    v, w = rng.standard_normal((B, T, H, V)), rng.random((B, T, H, V))
    a, e = rng.uniform(0.6, 1.0, (B, T, H, K)), rng.random((B, T, H, K))
    valid = rng.random((B, T)) > 0.1
    reset = rng.random((B, T)) > 0.93
    init = 0.1 * rng.standard_normal((B, H, K, V))
    go, gf, gs = rng.standard_normal((B, T, H, V)), rng.standard_normal((B, H, K, V)), rng.standard_normal((B, T, H))
    d = lambda x: torch.as_tensor(np.asarray(x, np.float32), device=cuda)  # noqa: E731
    args = [d(x) for x in (q, k, v, a, e, w, valid, reset, init)]
    plain = dbl.gdn_training_scan(*args, chunk)
    saved, ctx = dbl.gdn_training_scan_saved(*args, chunk)
    torch.cuda.synchronize()
    assert (ctx.numel() > 0) == (chunk == 16)
    f64 = [np.asarray(x, np.float32) for x in (q, k, v, a, e, w)]
    out, fin, sco = O.scan(*f64, valid, reset, np.asarray(init, np.float32))
    for got, ref_plain, ref in ((saved.output, plain.output, out), (saved.final_state, plain.final_state, fin),
                                (saved.scores[..., 0], plain.scores[..., 0], sco)):
        assert rel_err(host(got), ref) < TOL_F32
        assert rel_err(host(got), host(ref_plain)) < TOL_F32
    g0 = dbl.gdn_training_backward(*args, d(go), d(gf), d(gs), chunk_size=chunk)
    g1 = dbl.gdn_training_backward_saved(*args, d(go), ctx, d(gf), d(gs), chunk_size=chunk)
    torch.cuda.synchronize()
    ref = O.training_backward(*f64, *(np.asarray(x, np.float32) for x in (go, gf, gs)), valid, reset,
                              np.asarray(init, np.float32))
    names = ("dq", "dk", "dv", "dalpha", "derase", "dwrite", "dinitial")
    for name, r in zip(names, ref):
        x0, x1 = getattr(g0, name).cpu().numpy(), getattr(g1, name).cpu().numpy()
        assert np.array_equal(x0, x1), name
        assert rel_err(x1, r) < TOL_F32, (name, rel_err(x1, r))


def test_training_scan_and_backward_in_a_cuda_graph(cuda, native_lib):
    # the chunked forward (its workspace a graph memory node while the stream is captured) and the
    # saved-context backward captured into one CUDA graph and replayed: the same outputs and
    # gradients as eager calls
    B, T, H, K, V = 2, 64, 3, 32, 64
    rng = np.random.default_rng(5)
    q, k = rng.standard_normal((B, T, H, K)) / np.sqrt(K), rng.standard_normal((B, T, H, K)) / np.sqrt(K)
    v, w = rng.standard_normal((B, T, H, V)), rng.random((B, T, H, V))
    a, e = rng.uniform(0.6, 1.0, (B, T, H, K)), rng.random((B, T, H, K))
    valid, reset = rng.random((B, T)) > 0.1, rng.random((B, T)) > 0.93
    init = 0.1 * rng.standard_normal((B, H, K, V))
    go, gf, gs = rng.standard_normal((B, T, H, V)), rng.standard_normal((B, H, K, V)), rng.standard_normal((B, T, H))
    d = lambda x: torch.as_tensor(np.asarray(x, np.float32), device=cuda)  # noqa: E731
    args = [d(x) for x in (q, k, v, a, e, w, valid, reset, init)]
    ups = [d(go), d(gf), d(gs)]

    def step():
        fwd = dbl.gdn_training_scan(*args, 16)
        res, ctx = dbl.gdn_training_scan_saved(*args, 16)
        grads = dbl.gdn_training_backward_saved(*args, ups[0], ctx, ups[1], ups[2], chunk_size=16)
        return fwd, res, grads

    eager = step()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        step()
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        captured = step()
    graph.replay()
    graph.replay()
    torch.cuda.synchronize()
    for x, y in ((eager[0].output, captured[0].output), (eager[0].scores, captured[0].scores),
                 (eager[1].output, captured[1].output), (eager[1].final_state, captured[1].final_state)):
        assert torch.equal(x, y)
    for name in ("dq", "dk", "dv", "dalpha", "derase", "dwrite", "dinitial"):
        assert torch.equal(getattr(eager[2], name), getattr(captured[2], name)), name


# ----------------------------------------------------------------------- mixer prologue
@pytest.mark.parametrize("B,T,H,K,V,W,dtype", [(2, 37, 3, 32, 64, 4, torch.float32),
                                                (1, 50, 2, 128, 128, 4, torch.bfloat16),
                                                (2, 9, 2, 40, 72, 1, torch.float32),
                                                (1, 20, 2, 36, 20, 3, torch.bfloat16),
                                                (1, 70, 1, 256, 256, 8, torch.float32)])
def test_gdn2_prologue_matches_oracle(cuda, native_lib, B, T, H, K, V, W, dtype):
    # lib.rs:446-528 (MixerKind::Gdn2): conv + silu + l2 for q, k; conv + silu for v; decay and
    # sigmoid gates -- against the f64 prologue oracle, with padding and resets in the documents.
    rng = np.random.default_rng(T + K)
    r = lambda *s: rng.standard_normal(s)  # noqa: E731
    proj = [r(B, T, H * K), r(B, T, H * K), r(B, T, H * V), 3 * r(B, T, H * K), r(B, T, H * K), r(B, T, H * V)]
    proj[3][0, 0, :3] = [30.0, 21.0, -25.0]  # both sides of the softplus threshold
    conv = [0.3 * r(W, H * K), 0.3 * r(W, H * K), 0.3 * r(W, H * V)]
    bias, scale = 0.5 * r(H * K), 0.3 * r(H)
    valid = (rng.random((B, T)) > 0.15).astype(np.float32)
    reset = (rng.random((B, T)) > 0.8).astype(np.float32)
    if dtype == torch.bfloat16:
        proj = [bf16_round(x) for x in proj]
    d = lambda x, dt=torch.float32: torch.as_tensor(np.asarray(x, np.float32), device=cuda).to(dt)  # noqa: E731
    got = dbl.gdn2_prologue(*(d(x, dtype) for x in proj), *(d(x) for x in conv), d(bias), d(scale), d(valid),
                            d(reset), heads=H, out_dtype=dtype)
    torch.cuda.synchronize()
    ref = O.gdn2_prologue(*proj, *conv, bias, scale, valid, reset, heads=H)
    # gates (f32, in [0, 1]): within 2e-6 absolute of the f64 oracle; q, k, v within 2e-5 relative
    # (elementwise, against |e| + rms) in f32, within bf16 rounding otherwise
    for name, g, e in zip(("q", "k", "v", "alpha", "erase", "write"), got, ref):
        g = g.float().cpu().numpy()
        if name in ("alpha", "erase", "write"):
            assert np.abs(g - e).max() < 2e-6, (name, np.abs(g - e).max())
        else:
            tol = TOL_BF16 if dtype == torch.bfloat16 else 2e-5
            assert rel_err(g, e) < tol, (name, rel_err(g, e))


# ----------------------------------------------------------------- reference-layout relay attention
def _packed_layout(docs_per_row, tokens):
    """Packed documents (dre-core lib.rs:105-175): ids across rows, inclusive limits; padding
    tokens have start = position, end = position - 1, id -1."""
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
    return di, ds, de, doc


def _relay_inputs(docs_per_row, tokens, heads, seed, dtype):
    rng = np.random.default_rng(seed)
    di, ds, de, nd = _packed_layout(docs_per_row, tokens)
    B = len(docs_per_row)
    q, k, v = (rng.standard_normal((B, heads, tokens, 64)) for _ in range(3))
    rk, rv = (rng.standard_normal((nd, heads, 16, 64)) for _ in range(2))
    if dtype == torch.bfloat16:
        q, k, v, rk, rv = (bf16_round(x) for x in (q, k, v, rk, rv))
    return q, k, v, rk, rv, di, ds, de


def _relay_run(cuda, dtype, q, k, v, rk, rv, di, ds, de):
    d = lambda x: torch.as_tensor(np.asarray(x, np.float32), device=cuda).to(dtype)  # noqa: E731
    i = lambda x: torch.as_tensor(x, device=cuda)  # noqa: E731
    o, norm = dbl.relay_attention_forward(d(q), d(k), d(v), d(rk), d(rv), i(di), i(ds), i(de))
    torch.cuda.synchronize()
    assert native_device_ok()
    return o.float().cpu().numpy(), norm.cpu().numpy()


def native_device_ok():
    code = ctypes.c_int(0)
    return N.lib().dbl_device_error(ctypes.byref(code)) == 0 and code.value == 0


def _relay_check(o, norm, eo, en, dtype):
    # f32: the reference's own tolerance, 2e-5 + 1e-4 |e| (relay.rs:166-171); bf16: P enters the
    # tensor cores as bf16, so o is within bf16 rounding of the f64 oracle
    if dtype == torch.float32:
        np.testing.assert_allclose(o, eo, rtol=1e-4, atol=2e-5)
        np.testing.assert_allclose(norm, en, rtol=1e-4, atol=2e-5)
    else:
        assert rel_err(o, eo) < 1e-2, rel_err(o, eo)
        np.testing.assert_allclose(norm[..., 0], en[..., 0], rtol=1e-5, atol=1e-4)
        np.testing.assert_allclose(norm[..., 1], en[..., 1], rtol=1e-4)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("docs,tokens,heads", [([[2, 3]], 6, 1),               # relay_tests.rs:94-140 layout
                                               ([[100, 57, 80], [300]], 300, 3),  # padding tails, 3 tiles
                                               ([[258]], 258, 2),               # window edges at radius 128
                                               ([[2] * 512], 1024, 2)])         # relay_tests.rs:244: 512 documents
def test_relay_attention_matches_oracle(cuda, native_lib, dtype, docs, tokens, heads):
    q, k, v, rk, rv, di, ds, de = _relay_inputs(docs, tokens, heads, tokens + heads, dtype)
    o, norm = _relay_run(cuda, dtype, q, k, v, rk, rv, di, ds, de)
    eo, en = O.relay_window(q, k, v, rk, rv, di, ds, de)
    _relay_check(o, norm, eo, en, dtype)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_relay_attention_extreme_scores(cuda, native_lib, dtype):
    # relay_tests.rs:12-93: scores near -8e32; one effective key gives exactly its value and (m, 1);
    # eighteen equal keys give the sum 18
    di, ds, de, _ = _packed_layout([[1]], 2)
    q = np.full((1, 1, 2, 64), 1e16)
    k = np.full((1, 1, 2, 64), -1e16)
    v = np.array([i - 32.0 if i < 64 else 17.0 for i in range(128)]).reshape(1, 1, 2, 64)
    o, norm = _relay_run(cuda, dtype, q, k, v, np.full((1, 1, 16, 64), -2e16), np.full((1, 1, 16, 64), 23.0),
                         di, ds, de)
    assert np.isfinite(norm[0, 0, 0, 0]) and norm[0, 0, 0, 0] < -1e30 and norm[0, 0, 0, 1] == 1.0
    assert list(norm[0, 0, 1]) == [0.0, 1.0]
    assert np.array_equal(o[0, 0, 0], v[0, 0, 0]) and np.all(o[0, 0, 1] == 0.0)
    di, ds, de, _ = _packed_layout([[2]], 2)
    o, norm = _relay_run(cuda, dtype, q, k, np.zeros_like(v), np.full((1, 1, 16, 64), -1e16),
                         np.zeros((1, 1, 16, 64)), di, ds, de)
    assert np.all(np.isfinite(norm[..., 0])) and np.all(norm[..., 0] < -1e30) and np.all(norm[..., 1] == 18.0)
    assert np.all(o == 0.0)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_relay_attention_ignores_nan_padding(cuda, native_lib, dtype):
    # relay.rs:173-210: NaN in padding tokens (and in padding documents' relay slots) leaves the
    # live outputs unchanged and finite
    docs, tokens = [[90, 60], [200]], 260
    q, k, v, rk, rv, di, ds, de = _relay_inputs(docs, tokens, 2, 5, dtype)
    clean = _relay_run(cuda, dtype, q, k, v, rk, rv, di, ds, de)
    pad = de < ds
    q2, k2, v2 = (x.copy() for x in (q, k, v))
    for x in (q2, k2, v2):
        x.transpose(0, 2, 1, 3)[pad] = np.nan
    rk2 = np.concatenate([rk, np.full((2,) + rk.shape[1:], np.nan)])
    rv2 = np.concatenate([rv, np.full((2,) + rv.shape[1:], np.nan)])
    dirty = _relay_run(cuda, dtype, q2, k2, v2, rk2, rv2, di, ds, de)
    assert np.all(np.isfinite(dirty[0])) and np.all(np.isfinite(dirty[1]))
    np.testing.assert_array_equal(dirty[0], clean[0])
    np.testing.assert_array_equal(dirty[1], clean[1])


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_relay_attention_all_padding_no_documents(cuda, native_lib, dtype):
    # a batch without documents (document capacity 0, relay tensors [0, H, 16, 64]): every row is
    # padding and gives o = 0 and (0, 1), as relay_attention_kernel.rs:113-123
    B, H, T = 2, 3, 150
    di, ds, de, nd = _packed_layout([[], []], T)
    assert nd == 0
    x = [torch.randn(B, H, T, 64, device=cuda).to(dtype) for _ in range(3)]
    r = [torch.zeros(0, H, 16, 64, device=cuda, dtype=dtype) for _ in range(2)]
    o, norm = dbl.relay_attention_forward(*x, *r, *(torch.as_tensor(a, device=cuda) for a in (di, ds, de)))
    torch.cuda.synchronize()
    assert native_device_ok()
    assert torch.all(o == 0) and torch.all(norm[..., 0] == 0) and torch.all(norm[..., 1] == 1)


def test_relay_attention_rejects_bad_shapes(cuda, native_lib):
    q = torch.zeros(1, 1, 4, 32, device=cuda)
    ids = torch.zeros(1, 4, dtype=torch.int32, device=cuda)
    with pytest.raises(ValueError):
        dbl.relay_attention_forward(q, q, q, torch.zeros(1, 1, 16, 32, device=cuda), torch.zeros(1, 1, 16, 32, device=cuda),
                                    ids, ids, ids)


# ------------------------------------------------------------------------- gdn2_scan backward
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("B,T,H", [(2, 45, 2), (1, 130, 3)])
def test_gdn2_scan_backward_matches_oracle(cuda, native_lib, dtype, B, T, H):
    # gdn2_backward (ops.rs:106-160, gdn2.rs:285-519) at the reference's widths K32 / V64, documents
    # with resets and a padding tail, against the f64 backward oracle on the same (rounded) inputs
    K, V = 32, 64
    rng = np.random.default_rng(T + H)
    q, k = rng.standard_normal((B, T, H, K)) / 6, rng.standard_normal((B, T, H, K)) / 6
    v, w = rng.standard_normal((B, T, H, V)), 1 / (1 + np.exp(-rng.standard_normal((B, T, H, V))))
    a = 1 / (1 + np.exp(-(3 + rng.standard_normal((B, T, H, K)))))
    e = 1 / (1 + np.exp(-rng.standard_normal((B, T, H, K))))
    go = rng.standard_normal((B, T, H, V))
    lengths = [[T // 3, T // 3], [T - 5]] if B == 2 else [[T // 2, T // 4]]
    di, ds, de, _ = _packed_layout(lengths, T)
    if dtype == torch.bfloat16:
        q, k, v, go = (bf16_round(x) for x in (q, k, v, go))
    d = lambda x, dt=torch.float32: torch.as_tensor(np.asarray(x, np.float32), device=cuda).to(dt)  # noqa: E731
    got = dbl.gdn2_scan_backward(d(q, dtype), d(k, dtype), d(v, dtype), d(a), d(e), d(w),
                                 torch.as_tensor(ds, device=cuda), torch.as_tensor(de, device=cuda), d(go, dtype))
    torch.cuda.synchronize()
    ref = O.doc_backward(q, k, v, a, e, w, ds, de, go)
    for name, g, r in zip(("dq", "dk", "dv", "dalpha", "derase", "dwrite"), got, ref):
        tol = TOL_BF16 if (dtype == torch.bfloat16 and name in ("dq", "dk", "dv")) else TOL_F32
        assert rel_err(g.float().cpu().numpy(), r) < tol, (name, rel_err(g.float().cpu().numpy(), r))
    # padding tokens get no gradient
    pad = (de < ds)
    for g in got:
        assert torch.all(g.float().cpu()[torch.as_tensor(pad)] == 0.0)


def test_prefill_from_host_matches_device(cuda, native_lib):
    # the host-buffer entry point (copies and kernels pipelined over batch slices on side streams)
    # gives the device path's results exactly: the sequences of a batch are independent
    B, T, H, D = 5, 192, 2, 128
    g = torch.Generator().manual_seed(21)
    q = torch.nn.functional.normalize(torch.randn(B, T, H, D, generator=g), dim=-1).bfloat16()
    k = torch.nn.functional.normalize(torch.randn(B, T, H, D, generator=g), dim=-1).bfloat16()
    v = torch.randn(B, T, H, D, generator=g).bfloat16()
    alpha = torch.sigmoid(3 + torch.randn(B, T, H, generator=g))
    beta = torch.sigmoid(torch.randn(B, T, H, generator=g))
    ref_o, ref_f = dbl.gdn2_prefill(*(x.to(cuda) for x in (q, k, v, alpha, beta)))
    ho, hf = dbl.gdn2_prefill_host(*(x.pin_memory() for x in (q, k, v, alpha, beta)), device=cuda, pieces=3)
    torch.cuda.synchronize()
    assert torch.equal(ho, ref_o.cpu()) and torch.equal(hf, ref_f.cpu())
    with pytest.raises(ValueError):
        dbl.gdn2_prefill_host(q.to(cuda), k, v, alpha, beta)


# ------------------------------------------------------------------------- single-token inputs
def test_single_token_inputs(cuda, native_lib):
    # T = 1 through the prologue (no conv history), relay attention (a window of one key plus the
    # relay slots) and the gdn2_scan backward (one token, one document), against the oracles
    rng = np.random.default_rng(5)
    H, K, V, W = 2, 32, 64, 4
    proj = [rng.standard_normal((1, 1, H * K)), rng.standard_normal((1, 1, H * K)), rng.standard_normal((1, 1, H * V)),
            rng.standard_normal((1, 1, H * K)), rng.standard_normal((1, 1, H * K)), rng.standard_normal((1, 1, H * V))]
    conv = [0.3 * rng.standard_normal((W, H * K)), 0.3 * rng.standard_normal((W, H * K)),
            0.3 * rng.standard_normal((W, H * V))]
    bias, scale = 0.5 * rng.standard_normal(H * K), 0.3 * rng.standard_normal(H)
    one, zero = np.ones((1, 1)), np.zeros((1, 1))
    d = lambda x: torch.as_tensor(np.asarray(x, np.float32), device=cuda)  # noqa: E731
    got = dbl.gdn2_prologue(*(d(x) for x in proj), *(d(x) for x in conv), d(bias), d(scale), d(one), d(zero), heads=H)
    ref = O.gdn2_prologue(*proj, *conv, bias, scale, one, zero, heads=H)
    for g, r in zip(got, ref):
        assert rel_err(g.cpu().numpy(), r) < 2e-5
    for dtype in (torch.float32, torch.bfloat16):
        q, k, v, rk, rv, di, ds, de = _relay_inputs([[1]], 1, H, 7, dtype)
        o, norm = _relay_run(cuda, dtype, q, k, v, rk, rv, di, ds, de)
        eo, en = O.relay_window(q, k, v, rk, rv, di, ds, de)
        _relay_check(o, norm, eo, en, dtype)
    q, k = rng.standard_normal((1, 1, H, K)) / 6, rng.standard_normal((1, 1, H, K)) / 6
    v, w = rng.standard_normal((1, 1, H, V)), rng.random((1, 1, H, V))
    a, e = rng.uniform(0.5, 1.0, (1, 1, H, K)), rng.random((1, 1, H, K))
    go = rng.standard_normal((1, 1, H, V))
    ds1, de1 = np.zeros((1, 1), np.int32), np.zeros((1, 1), np.int32)
    got = dbl.gdn2_scan_backward(*(d(x) for x in (q, k, v, a, e, w)), torch.as_tensor(ds1, device=cuda),
                                 torch.as_tensor(de1, device=cuda), d(go))
    ref = O.doc_backward(q, k, v, a, e, w, ds1, de1, go)
    for g, r in zip(got, ref):
        assert rel_err(g.cpu().numpy(), r) < TOL_F32


# --------------------------------------------------------------- full-size, size-independent checks
def test_prefill_full_size_linear_in_values_and_permutation(cuda, native_lib):
    # BASELINE config 1 (B8/H16/T4096/d128 bf16) for every head: the output and final state are
    # linear in v for a zero initial state, so doubling v doubles them.  The kernel is deterministic
    # (the same inputs give the same bits) and each (b, h) is computed on its own (permuting the batch
    # permutes the results bit for bit).  Doubling is exact in floating point except for fp16 MMA
    # operands below fp16's normal range (6.1e-5: a decay-scaled edit of a strongly decayed token),
    # which round on a different grid once doubled; that moves outputs by about 1e-3 of their rms at
    # a handful of near-zero elements and can flip an output's bf16 rounding, so linearity is held to
    # one bf16 unit plus 2e-3 rms (outputs) and 1e-3 of the soft metric (final states).
    import bench
    q, k, v, alpha, beta = bench.make_prefill_inputs(torch, cuda, 4321)
    o1, f1 = dbl.gdn2_prefill(q, k, v, alpha, beta)
    o1b, f1b = dbl.gdn2_prefill(q, k, v, alpha, beta)
    o2, f2 = dbl.gdn2_prefill(q, k, v * 2, alpha, beta)
    perm = torch.tensor([3, 0, 7, 1, 6, 2, 5, 4], device=cuda)
    o3, f3 = dbl.gdn2_prefill(q[perm], k[perm], v[perm], alpha[perm], beta[perm])
    torch.cuda.synchronize()
    assert _device_error_clear(native_lib) == (0, 0)
    # deterministic: the same inputs give the same bits
    assert torch.equal(o1b, o1) and torch.equal(f1b, f1), int((o1b != o1).sum())
    assert torch.equal(o3, o1[perm]) and torch.equal(f3, f1[perm])
    assert torch.isfinite(o1.float()).all() and torch.isfinite(f1).all()
    # one bf16 unit of the element (a flipped output rounding) plus 2e-3 of the rms (near-zero
    # outputs, where the shifted subnormal roundings of the operands are not small relative to |o|)
    a2, e2 = host(o2.float()), 2 * host(o1.float())
    rms = float(np.sqrt(np.mean(e2 * e2)))
    excess = np.abs(a2 - e2) - (2.0 ** -7 * np.abs(e2) + 2e-3 * rms)
    worst = np.unravel_index(np.argmax(excess), excess.shape)
    assert excess[worst] <= 0, (worst, float(a2[worst]), float(e2[worst]), rms)
    assert rel_err(host(f2), 2 * host(f1)) < 1e-3


def test_prologue_full_size_sampled(cuda, native_lib):
    # the prologue at the config-1 shape (B8/T4096/H16, K = V = 128, bf16), three (b, head, token
    # window) slices against the oracle, each window with its conv history
    b_, t_, h_, d = 8, 4096, 16, 128
    g = torch.Generator(device=cuda)
    g.manual_seed(13)
    proj = [torch.randn(b_, t_, h_ * d, device=cuda, generator=g).bfloat16() for _ in range(6)]
    conv = [0.3 * torch.randn(4, h_ * d, device=cuda, generator=g) for _ in range(3)]
    bias, scale = torch.randn(h_ * d, device=cuda, generator=g), 0.3 * torch.randn(h_, device=cuda, generator=g)
    valid = torch.ones(b_, t_, device=cuda)
    reset = (torch.rand(b_, t_, device=cuda, generator=g) > 0.99).float()
    got = dbl.gdn2_prologue(*proj, *conv, bias, scale, valid, reset, heads=h_, out_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    for b, h, t0 in ((0, 0, 0), (5, 11, 2000), (7, 15, 4096 - 200)):
        lo, hi = max(0, t0 - 8), min(t_, t0 + 200)
        cols = slice(h * d, (h + 1) * d)
        ref = O.gdn2_prologue(*(host(x[b:b + 1, lo:hi, cols]) for x in proj), *(host(c[:, cols]) for c in conv),
                              host(bias[cols]), host(scale[h:h + 1]), host(valid[b:b + 1, lo:hi]),
                              host(reset[b:b + 1, lo:hi]), heads=1)
        # the first rows of the window lack their conv history unless the window starts at t = 0
        skip = 0 if lo == 0 else 8
        for gi, r in zip(got, ref):
            g_slice = host(gi[b:b + 1, lo:hi, h:h + 1].float())
            tol = 2e-6 if gi.dtype == torch.float32 else TOL_BF16
            if gi.dtype == torch.float32:
                assert np.abs(g_slice[:, skip:] - r[:, skip:]).max() < tol
            else:
                assert rel_err(g_slice[:, skip:], r[:, skip:]) < tol


def test_relay_attention_full_size_sampled(cuda, native_lib):
    # reference-layout relay attention at the bench shape (B8/H16/T4096, 1024-token documents,
    # bf16): three (b, h) heads against the oracle, and every row finite
    b_, h_, t_, dl = 8, 16, 4096, 1024
    nd = b_ * t_ // dl
    g = torch.Generator(device=cuda)
    g.manual_seed(17)
    x = [torch.randn(b_, h_, t_, 64, device=cuda, generator=g).bfloat16() for _ in range(3)]
    r = [torch.randn(nd, h_, 16, 64, device=cuda, generator=g).bfloat16() for _ in range(2)]
    pos = torch.arange(t_, device=cuda, dtype=torch.int32)
    ds = (pos // dl * dl).expand(b_, t_).contiguous()
    de = (ds + dl - 1).contiguous()
    di = (torch.arange(b_, device=cuda, dtype=torch.int32)[:, None] * (t_ // dl) + pos // dl).contiguous()
    o, norm = dbl.relay_attention_forward(*x, *r, di, ds, de)
    torch.cuda.synchronize()
    assert native_device_ok()
    assert torch.isfinite(o.float()).all() and torch.isfinite(norm).all()
    for b, h in ((0, 0), (3, 9), (7, 15)):
        # the head's documents are b * 4 .. b * 4 + 3 (relay slots of this head only)
        eo, en = O.relay_window(*(host(t[b:b + 1, h:h + 1].float()) for t in x),
                                *(host(t[4 * b:4 * b + 4, h:h + 1].float()) for t in r),
                                host(di[b:b + 1]) - 4 * b, host(ds[b:b + 1]), host(de[b:b + 1]))
        _relay_check(host(o[b:b + 1, h:h + 1].float()), host(norm[b:b + 1, h:h + 1]), eo, en, torch.bfloat16)
