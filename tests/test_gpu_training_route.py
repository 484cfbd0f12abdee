"""The reference's drop-in call, gdn_training_scan (crates/kernels/src/gdn_training_ops.rs:288-333),
at K = V = 128 with bf16 inputs: every (b, h) whose gates are constant across channels runs on the
tensor-core kernel, every other one on the token-sequential kernel, in one call with no host
synchronisation.  Checked against the f64 oracle (outputs, final states, scores), including a
call that mixes both kinds of (b, h) and one with different erase and write gates.
"""
import numpy as np
import pytest
import torch

import delta_block_lm_b200 as dbl
from fixtures import TOL_BF16, TOL_F32, baseline_inputs, bf16_round, rel_err, report
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def dev_t(x, device, dtype=torch.float32):
    return torch.as_tensor(np.ascontiguousarray(x), dtype=torch.float32).to(device=device, dtype=dtype)


def host(t):
    return t.detach().float().cpu().numpy()


def _case(seed, B, T, H, D, erase_scale=1.0, varying=()):
    q, k, v, alpha, beta = baseline_inputs(seed, B, T, H, D, D)
    q = bf16_round(q / np.sqrt(D))
    k, v = bf16_round(k), bf16_round(v)
    a = np.repeat(alpha[..., None], D, 3)
    e = np.repeat((erase_scale * beta)[..., None], D, 3).astype(np.float32)
    w = np.repeat(beta[..., None], D, 3)
    rng = np.random.default_rng(seed + 7)
    for b, h in varying:  # channel-wise gates on these (b, h): the token-sequential kernel's rows
        a[b, :, h] = (1 / (1 + np.exp(-(3 + rng.standard_normal((T, D)))))).astype(np.float32)
        e[b, :, h] = (1 / (1 + np.exp(-rng.standard_normal((T, D))))).astype(np.float32)
    valid = rng.random((B, T)) > 0.05
    reset = rng.random((B, T)) > 0.98
    init = (0.02 * rng.standard_normal((B, H, D, D))).astype(np.float32)
    return q, k, v, a, e, w, valid, reset, init


@pytest.mark.parametrize("erase_scale,varying", [(1.0, ()), (0.7, ()), (1.0, ((0, 1), (1, 2)))])
def test_training_scan_routed_matches_oracle(cuda, native_lib, erase_scale, varying):
    B, T, H, D = 2, 300, 3, 128
    q, k, v, a, e, w, valid, reset, init = _case(3, B, T, H, D, erase_scale, varying)
    bf = lambda x: dev_t(x, cuda, torch.bfloat16)  # noqa: E731
    r = dbl.gdn_training_scan(bf(q), bf(k), bf(v), dev_t(a, cuda), dev_t(e, cuda), dev_t(w, cuda),
                              dev_t(valid, cuda), dev_t(reset, cuda), dev_t(init, cuda), 16)
    torch.cuda.synchronize()
    ro, rf, rs = O.scan(q, k, v, a, e, w, valid, reset, init)
    rep = report(f"gdn_training_scan routed bf16 d128, erase x{erase_scale}, channel-wise rows {list(varying)}",
                 out=(host(r.output), ro), final_state=(host(r.final_state), rf), scores=(host(r.scores)[..., 0], rs))
    for name in ("out", "final_state", "scores"):
        assert rep[name]["rel_err"] < TOL_BF16, name
    assert np.all(host(r.output)[~valid] == 0.0) and np.all(host(r.scores)[..., 0][~valid] == 0.0)
    # the (b, h) rows with channel-wise gates ran on the f32 token-sequential kernel: reference bound
    for b, h in varying:
        assert rel_err(host(r.output)[b, :, h], ro[b, :, h]) < TOL_F32, (b, h)
