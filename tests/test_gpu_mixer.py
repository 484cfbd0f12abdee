"""GPU tests of the mixer-side entry point scan_selected (crates/mixers/src/chunk.rs:29-108).

Both fused backends are run against the f64 oracle through the call the mixers crate makes:
  * FUSED_GDN2 on the reference's sinusoidal + edge-edit fixture (checks.rs:119-180,
    kron_checks.rs:132-175), channel-wise gates, valid / reset, initial state, scores;
  * CHUNKED_GDN2 (scalar gates, q pre-scaled: scale 1.0) at bf16 K = V = 128 with masks and an
    initial state, i.e. the tensor-core kernel behind the selector;
  * the decode step as the reference writes it: T = 1 with ``initial`` = the state after a prefix
    (crates/mixers/src/lib.rs:544-556), for both backends, compared with the oracle's last token.
"""
import numpy as np
import pytest
import torch

from delta_block_lm_b200.mixers import MixerKind, ScanBackend, ScanInput, scan_selected
from fixtures import (TOL_BF16, baseline_inputs, bf16_round, edge_edits, edge_initial, ref_close, report,
                      sinusoid_fixture)
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def dev_t(x, device, dtype=torch.float32):
    return torch.as_tensor(np.ascontiguousarray(x), dtype=torch.float32).to(device=device, dtype=dtype)


def host(t):
    return t.detach().float().cpu().numpy()


@pytest.mark.parametrize("t", [7, 35])
def test_fused_gdn2_edge_fixture(cuda, native_lib, t):
    fields, valid, reset = sinusoid_fixture(t)
    fields, valid, reset = edge_edits(fields, valid, reset)
    init = edge_initial()
    inp = ScanInput(*[dev_t(x, cuda) for x in fields])
    r = scan_selected(ScanBackend.FUSED_GDN2, MixerKind.GDN2, inp, dev_t(valid, cuda), dev_t(reset, cuda), 16,
                      dev_t(init, cuda))
    torch.cuda.synchronize()
    ro, rf, rs = O.scan(*fields, valid, reset, init)
    report(f"scan_selected FUSED_GDN2 edge fixture T{t}", out=(host(r.output), ro),
           final_state=(host(r.final_state), rf), scores=(host(r.scores)[..., 0], rs))
    for got, exp in ((r.output, ro), (r.final_state, rf), (r.scores[..., 0], rs)):
        ok, err = ref_close(host(got), exp)
        assert ok, err


def _scalar_case(cuda, seed, B, T, H, D):
    q, k, v, alpha, beta = baseline_inputs(seed, B, T, H, D, D)
    q = q / np.sqrt(D)  # CHUNKED_GDN2 takes q pre-scaled (scale 1.0)
    q, k, v = bf16_round(q), bf16_round(k), bf16_round(v)
    rng = np.random.default_rng(seed + 1)
    valid = rng.random((B, T)) > 0.05
    reset = rng.random((B, T)) > 0.98
    init = (0.02 * rng.standard_normal((B, H, D, D))).astype(np.float32)
    return q, k, v, alpha, beta, valid, reset, init


def test_chunked_gdn2_bf16_d128(cuda, native_lib):
    B, T, H, D = 2, 300, 2, 128
    q, k, v, alpha, beta, valid, reset, init = _scalar_case(cuda, 3, B, T, H, D)
    bf = lambda x: dev_t(x, cuda, torch.bfloat16)  # noqa: E731
    inp = ScanInput(bf(q), bf(k), bf(v), dev_t(alpha[..., None], cuda), dev_t(beta[..., None], cuda),
                    dev_t(beta[..., None], cuda))
    r = scan_selected(ScanBackend.CHUNKED_GDN2, MixerKind.GDN2, inp, dev_t(valid, cuda), dev_t(reset, cuda), 16,
                      dev_t(init, cuda))
    torch.cuda.synchronize()
    ro, rf, _ = O.scan_scalar(q, k, v, alpha, beta, valid, reset, init, scale=1.0)
    rep = report("scan_selected CHUNKED_GDN2 bf16 d128", out=(host(r.output), ro), final_state=(host(r.final_state), rf))
    assert rep["out"]["rel_err"] < TOL_BF16 and rep["final_state"]["rel_err"] < TOL_BF16
    assert np.all(host(r.output)[~valid] == 0.0)


def test_chunked_gdn2_gate_check_is_opt_in(cuda, native_lib):
    B, T, H, D = 1, 64, 1, 128
    q, k, v, alpha, beta, valid, reset, init = _scalar_case(cuda, 4, B, T, H, D)
    bf = lambda x: dev_t(x, cuda, torch.bfloat16)  # noqa: E731
    inp = ScanInput(bf(q), bf(k), bf(v), dev_t(alpha[..., None], cuda), dev_t(beta[..., None], cuda),
                    dev_t(0.5 * beta[..., None], cuda))
    with pytest.raises(ValueError):
        scan_selected(ScanBackend.CHUNKED_GDN2, MixerKind.GDN2, inp, dev_t(valid, cuda), dev_t(reset, cuda), 16,
                      dev_t(init, cuda), check_gates=True)


@pytest.mark.parametrize("backend", [ScanBackend.FUSED_GDN2, ScanBackend.CHUNKED_GDN2])
def test_decode_as_continuation(cuda, native_lib, backend):
    # the prefix [0, T-1) runs as one scan, its final state seeds a T = 1 call for the last token
    B, T, H, D = 2, 129, 2, 128
    q, k, v, alpha, beta, valid, reset, init = _scalar_case(cuda, 5, B, T, H, D)
    valid[:, -1] = True
    ro, rf, _ = O.scan_scalar(q, k, v, alpha, beta, valid, reset, init, scale=1.0)
    dt = torch.bfloat16

    def inputs(sl):
        qq, kk, vv = (dev_t(x[:, sl], cuda, dt) for x in (q, k, v))
        if backend == ScanBackend.FUSED_GDN2:
            a = dev_t(np.repeat(alpha[:, sl, :, None], D, 3), cuda)
            e = dev_t(np.repeat(beta[:, sl, :, None], D, 3), cuda)
            return ScanInput(qq, kk, vv, a, e, e.clone())
        return ScanInput(qq, kk, vv, dev_t(alpha[:, sl, :, None], cuda), dev_t(beta[:, sl, :, None], cuda),
                         dev_t(beta[:, sl, :, None], cuda))

    pre = scan_selected(backend, MixerKind.GDN2, inputs(slice(0, T - 1)), dev_t(valid[:, :T - 1], cuda),
                        dev_t(reset[:, :T - 1], cuda), 16, dev_t(init, cuda))
    last = scan_selected(backend, MixerKind.GDN2, inputs(slice(T - 1, T)), dev_t(valid[:, T - 1:], cuda),
                         dev_t(reset[:, T - 1:], cuda), 16, pre.final_state)
    torch.cuda.synchronize()
    rep = report(f"scan_selected {backend.value} decode as T=1 continuation",
                 out=(host(last.output)[:, 0], ro[:, T - 1]), final_state=(host(last.final_state), rf))
    assert rep["out"]["rel_err"] < TOL_BF16 and rep["final_state"]["rel_err"] < TOL_BF16
