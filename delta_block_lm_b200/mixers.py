"""Host mirror of the mixers crate's scan selector (crates/mixers/src/chunk.rs:8-108, lib.rs:40-85).

``scan_selected(backend, kind, input, valid, reset, chunk_size, initial)`` keeps the reference's
signature and dispatch rules: the fused backend requires GDN-2 and a GPU device and never falls
back (chunk.rs:110-124).  ``ScanBackend.CHUNKED_GDN2`` is the tensor-core chunked path for scalar
gates (alpha/erase/write of width 1 with erase == write, i.e. the BASELINE recurrence).
``ScanBackend.TENSOR_SOLVER`` names the reference's Burn tensor-op path, which this build does not
carry: selecting it raises instead of silently running something else.
"""
from __future__ import annotations

import enum
from dataclasses import dataclass
from typing import Optional

import torch

from . import kernels


class MixerKind(enum.Enum):
    GDN2 = "gdn2"
    KRON_LSTM = "kron_lstm"


class ScanBackend(enum.Enum):
    TENSOR_SOLVER = "tensor_solver"
    FUSED_GDN2 = "fused_gdn2"
    CHUNKED_GDN2 = "chunked_gdn2"

    def supports(self, kind: MixerKind) -> bool:
        return kind == MixerKind.GDN2

    def is_fused(self) -> bool:
        return self != ScanBackend.TENSOR_SOLVER


@dataclass
class ScanInput:
    q: torch.Tensor
    k: torch.Tensor
    v: torch.Tensor
    alpha: torch.Tensor
    erase: torch.Tensor   # channel-wise erase [B,T,H,K] (width 1 for scalar gates)
    write: torch.Tensor   # channel-wise write [B,T,H,V] (width 1 for scalar gates)


@dataclass
class ScanOutput:
    output: torch.Tensor
    final_state: torch.Tensor
    scores: Optional[torch.Tensor]  # norm of the active edit after decay; None on CHUNKED_GDN2


def assert_fused_device(device: torch.device) -> None:
    if device.type != "cuda":
        raise RuntimeError("fused GPU scan requires a CUDA GPU device; no CPU fallback")


def scan_selected(backend: ScanBackend, kind: MixerKind, input: ScanInput, valid: torch.Tensor,
                  reset: torch.Tensor, chunk_size: int, initial: Optional[torch.Tensor] = None,
                  *, check_gates: bool = False) -> ScanOutput:
    """Explicit dispatch; requesting fused execution never falls back to tensor operations.

    ``CHUNKED_GDN2`` takes ``erase`` as the scalar beta of the delta rule and requires
    ``write == erase``; that equality is the caller's contract and is not checked by default,
    because checking it reads both tensors back to the host (a device synchronisation per call).
    ``check_gates=True`` checks it and raises ``ValueError`` on a mismatch.  The decode step is
    this call with T = 1 and ``initial`` set (crates/mixers/src/lib.rs:544-556)."""
    if backend == ScanBackend.TENSOR_SOLVER:
        raise NotImplementedError(
            "tensor_solver is the reference's Burn tensor-op path; this build provides "
            "fused_gdn2 and chunked_gdn2 only")
    if kind != MixerKind.GDN2:
        raise ValueError(f"{backend.value} requires GDN-2")
    assert_fused_device(input.q.device)
    B, _, H, K = input.q.shape
    V = input.v.shape[3]
    if initial is None:
        initial = torch.zeros((B, H, K, V), device=input.q.device, dtype=torch.float32)
    if backend == ScanBackend.FUSED_GDN2:
        r = kernels.gdn_training_scan(input.q, input.k, input.v, input.alpha, input.erase,
                                      input.write, valid, reset, initial, chunk_size)
        return ScanOutput(r.output, r.final_state, r.scores)
    # CHUNKED_GDN2: scalar gates
    if input.alpha.shape[3] != 1 or input.erase.shape[3] != 1 or input.write.shape[3] != 1:
        raise ValueError("chunked_gdn2 requires scalar gates (alpha, erase, write of width 1)")
    beta = input.erase[..., 0].to(torch.float32)
    if check_gates and not torch.equal(beta, input.write[..., 0].to(torch.float32)):
        raise ValueError("chunked_gdn2 requires erase == write (the scalar beta of the delta rule)")
    out, final = kernels.gdn2_prefill(input.q, input.k, input.v,
                                      input.alpha[..., 0].to(torch.float32).contiguous(),
                                      beta.contiguous(), scale=1.0, valid=valid, reset=reset,
                                      initial_state=initial, chunk_size=64)
    return ScanOutput(out, final, None)
