"""CPU tests of the host-side mirror: dispatch rules and validation (no kernel is launched)."""
import pytest
import torch

import delta_block_lm_b200 as dbl
from delta_block_lm_b200.mixers import MixerKind, ScanBackend, ScanInput


def _input(B=1, T=4, H=2, K=8, V=8, width=None, device="cpu"):
    kw = K if width is None else width
    vw = V if width is None else width
    z = lambda *s: torch.zeros(*s, device=device)
    return ScanInput(z(B, T, H, K), z(B, T, H, K), z(B, T, H, V), z(B, T, H, kw), z(B, T, H, kw),
                     z(B, T, H, vw))


def test_tensor_solver_is_not_silently_substituted():
    with pytest.raises(NotImplementedError, match="tensor_solver"):
        dbl.scan_selected(ScanBackend.TENSOR_SOLVER, MixerKind.GDN2, _input(), torch.ones(1, 4),
                          torch.zeros(1, 4), 16)


def test_fused_requires_gdn2():
    with pytest.raises(ValueError, match="requires GDN-2"):
        dbl.scan_selected(ScanBackend.FUSED_GDN2, MixerKind.KRON_LSTM, _input(), torch.ones(1, 4),
                          torch.zeros(1, 4), 16)


def test_no_cpu_fallback():
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        dbl.scan_selected(ScanBackend.FUSED_GDN2, MixerKind.GDN2, _input(), torch.ones(1, 4),
                          torch.zeros(1, 4), 16)
    with pytest.raises(ValueError, match="no CPU fallback"):
        dbl.gdn2_prefill(torch.zeros(1, 4, 1, 8), torch.zeros(1, 4, 1, 8), torch.zeros(1, 4, 1, 8),
                         torch.ones(1, 4, 1), torch.ones(1, 4, 1))
    with pytest.raises(ValueError, match="no CPU fallback"):
        dbl.relay_merge_decode(torch.zeros(1, 1, 64), torch.zeros(1, 4, 64), torch.zeros(1, 4, 64),
                               torch.zeros(1, 1, 4, 64), torch.zeros(1, 1, 4, 64))


def test_backend_properties():
    assert ScanBackend.FUSED_GDN2.is_fused() and not ScanBackend.TENSOR_SOLVER.is_fused()
    assert ScanBackend.CHUNKED_GDN2.supports(MixerKind.GDN2)
