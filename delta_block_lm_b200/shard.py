"""Multi-GPU drivers of the GDN-2 prefill: one process per GPU, torch.distributed for the plumbing.

* Batch x head sharding: the (b, h) pairs are independent, so every rank runs
  ``kernels.gdn2_prefill`` on its own rows with no data-path collective (``shard_batch``).
* Time sharding of one long sequence: rank g holds the contiguous token span
  g of the sequence.  Over a span the state map is affine, S_end = A_g S_start + B_g, with A_g a
  K x K matrix per head (``kernels.gdn2_span_transition``) and B_g the scan of the span from a
  zero state.  The hand-off is one ``all_gather`` of the per-rank boundary objects (the only
  collective), after which each rank composes the maps of the ranks before it and rescans its
  span from its exact start state:
      rank 0     : scans its span from the true initial state; its final state is S_in(1)
      rank g > 0 : A_g, B_g from its span; S_in(g) = A_{g-1}(...(A_1 S_in(1) + B_1)...) + B_{g-1};
                   then the scan from S_in(g) gives its outputs and final state.
  The reference has no multi-device code; this module is the B200 build's own.
"""
from __future__ import annotations

from typing import List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist

from . import kernels


def shard_bounds(n: int, world: int, rank: int, align: int = 1) -> Tuple[int, int]:
    """[start, end) of rank's contiguous share of n items, cut on multiples of `align`."""
    units = (n + align - 1) // align
    lo = (units * rank) // world
    hi = (units * (rank + 1)) // world
    return min(n, lo * align), min(n, hi * align)


def shard_batch(q, k, v, alpha, beta, *, group=None, **kw):
    """Prefill of this rank's rows of a batch sharded over ranks (no collective)."""
    return kernels.gdn2_prefill(q, k, v, alpha, beta, **kw)


def fold_span_states(first_state: torch.Tensor, transitions: Sequence[torch.Tensor],
                     offsets: Sequence[torch.Tensor], upto: int) -> torch.Tensor:
    """S_in(upto) from S_in(1) = first_state and the spans 1 .. upto-1:
    S_in(g + 1) = A_g S_in(g) + B_g  (A_g [B,H,K,K], B_g / states [B,H,K,V], f32)."""
    s = first_state
    for g in range(1, upto):
        s = torch.matmul(transitions[g], s) + offsets[g]
    return s


def exchange_span_states(first_or_transition: torch.Tensor, offset: Optional[torch.Tensor],
                         rank: int, world: int, group=None
                         ) -> Tuple[List[torch.Tensor], List[torch.Tensor]]:
    """All-gather the boundary objects.  Rank 0 contributes its final state (S_in(1)) in the
    `offset` slot and no transition; rank g > 0 contributes (A_g, B_g).  Returns the lists
    (transitions, offsets) indexed by rank, with offsets[0] = S_in(1)."""
    if rank == 0:
        K = first_or_transition.shape[-2]
        A = torch.zeros(first_or_transition.shape[:-2] + (K, K), dtype=first_or_transition.dtype,
                        device=first_or_transition.device)
        Bv = first_or_transition
    else:
        A, Bv = first_or_transition, offset
    As = [torch.empty_like(A) for _ in range(world)]
    Bs = [torch.empty_like(Bv) for _ in range(world)]
    dist.all_gather(As, A.contiguous(), group=group)
    dist.all_gather(Bs, Bv.contiguous(), group=group)
    return As, Bs


def time_sharded_prefill(q, k, v, alpha, beta, *, group=None, scale: Optional[float] = None,
                         initial_state: Optional[torch.Tensor] = None, chunk_size: int = 64
                         ) -> Tuple[torch.Tensor, torch.Tensor]:
    """Prefill of one rank's time span of a sequence sharded along time.

    q, k, v [B, T_span, H, D] and alpha, beta [B, T_span, H] are this rank's contiguous span (rank
    order = time order; spans should be multiples of the 64-token chunk for best efficiency).
    ``initial_state`` is the sequence's initial state and is used by rank 0 only.  Returns this
    rank's outputs [B, T_span, H, V] and the state at the end of its span (on the last rank: the
    sequence's final state).
    """
    rank = dist.get_rank(group)
    world = dist.get_world_size(group)
    if world == 1:
        return kernels.gdn2_prefill(q, k, v, alpha, beta, scale=scale, initial_state=initial_state,
                                    chunk_size=chunk_size)
    if rank == 0:
        out, fin = kernels.gdn2_prefill(q, k, v, alpha, beta, scale=scale,
                                        initial_state=initial_state, chunk_size=chunk_size)
        exchange_span_states(fin, None, rank, world, group)
        return out, fin
    A = kernels.gdn2_span_transition(k, alpha, beta, chunk_size=chunk_size)
    _, Bspan = kernels.gdn2_prefill(q, k, v, alpha, beta, scale=scale, want_output=False,
                                    chunk_size=chunk_size)
    As, Bs = exchange_span_states(A, Bspan, rank, world, group)
    s_in = fold_span_states(Bs[0], As, Bs, rank)
    return kernels.gdn2_prefill(q, k, v, alpha, beta, scale=scale, initial_state=s_in,
                                chunk_size=chunk_size)
