"""Multi-GPU drivers of the GDN-2 prefill: one process per GPU, torch.distributed for the plumbing.

* Batch x head sharding: the (b, h) pairs are independent, so every rank runs
  ``kernels.gdn2_prefill`` on its own rows with no data-path collective (``shard_batch``).
* Time sharding of one long sequence.  Over a token span the state map is
  affine, S_end = A S_start + B, with A a K x K matrix per head (``kernels.gdn2_span_transition``)
  and B the scan of the span from a zero state.  A long span is cut into S segments that run as a
  batch (a strided [S, T/S, H, D] view of the same memory, so S x H CTAs fill the GPU):
      pass 1  all segment maps (A_s, B_s) in two batched launches;
      fold    the start state of every segment by composing the maps before it (one small
              kernel, dbl_gdn2_span_fold);
      pass 2  every segment rescanned from its exact start state in one batched launch.
  On one device the whole span is one C-ABI call (dbl_gdn2_prefill_segmented), whose default
  schedule scans a lead segment from the initial state beside the maps of the other segments.
  Across GPUs, rank g holds the contiguous span g; the ranks exchange their composed span maps
  with one ``all_gather`` (the only collective) and each rank folds the maps of the ranks before it
  into its own start state before the local fold.
The reference has no multi-device or time-parallel code; this module is the B200 build's own.
"""
from __future__ import annotations

from typing import List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist

from . import kernels

CHUNK = 64


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
    S_in(g + 1) = A_g S_in(g) + B_g  (A_g [B,H,K,K], B_g / states [B,H,K,V], f32).  On CUDA
    tensors this is one fold kernel (kernels.gdn2_span_fold); on CPU tensors (the gloo tests) the
    same recurrence in torch."""
    if upto <= 1:
        return first_state
    if first_state.is_cuda:
        A = torch.stack([transitions[g][0] for g in range(1, upto)])
        Bm = torch.stack([offsets[g][0] for g in range(1, upto)])
        _, end, _ = kernels.gdn2_span_fold(A, Bm, first_state[0])
        return end.unsqueeze(0)
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
    # one collective: each rank's (A_g | B_g) side by side, [.., K, K + V]
    K = A.shape[-1]
    packed = torch.cat([A, Bv], dim=-1).contiguous()
    parts = [torch.empty_like(packed) for _ in range(world)]
    dist.all_gather(parts, packed, group=group)
    return [x[..., :K] for x in parts], [x[..., K:] for x in parts]


def sm_count(device: Optional[torch.device] = None) -> int:
    """Streaming multiprocessors of `device` (the current CUDA device by default; 148 on a B200)."""
    if not torch.cuda.is_available():
        return 148
    return torch.cuda.get_device_properties(device if device is not None else torch.cuda.current_device()
                                            ).multi_processor_count


def pick_segments(t_span: int, heads: int, sms: int = 148) -> int:
    """Segments per span: the largest power of two with segments x heads <= sms whose segments are
    whole 64-token chunks (1 when the span is short or heads alone fill the GPU).  `sms` is the
    device's SM count (``sm_count``).  The C library's rule for equal segments when its lead
    schedule does not apply, and for its multi-device entry; the drivers here use
    ``segment_groups``."""
    s = 1
    while (s * 2) * heads <= sms and t_span % (s * 2 * CHUNK) == 0:
        s *= 2
    return s


def segment_groups(t_span: int, heads: int, sms: int = 148) -> List[Tuple[int, int, int]]:
    """The segments of one span as groups (t0, count, length): `count` consecutive segments of
    `length` tokens from token t0.  Up to floor(sms / heads) segments of ceil(chunks / that) whole
    64-token chunks, so one launch of segments x heads CTAs fills the device; when the chunks do
    not divide evenly the last segment is shorter and forms a second group (a second, concurrent
    launch).  A span that is not whole chunks is one segment."""
    if t_span % CHUNK:
        return [(0, 1, t_span)]
    n = t_span // CHUNK
    m = max(1, min(sms // max(1, heads), n))
    L = -(-n // m)
    full = n // L
    groups = [(0, full, L * CHUNK)]
    if n > full * L:
        groups.append((full * L * CHUNK, 1, (n - full * L) * CHUNK))
    return groups


def _resolve_groups(t_span: int, heads: int, device, segments: Optional[int]):
    """`segments` equal segments when given (None when they do not divide the span), else
    segment_groups for the device."""
    if segments:
        return [(0, segments, t_span // segments)] if t_span % segments == 0 else None
    return segment_groups(t_span, heads, sm_count(device))


def _group_view(x: torch.Tensor, t0: int, count: int, length: int) -> torch.Tensor:
    """Tokens [t0, t0 + count * length) of [1, T, ...] as [count, length, ...] (same memory)."""
    return x[:, t0:t0 + count * length].reshape((count, length) + tuple(x.shape[2:]))


_SIDE = {}


def _on_groups(groups, fn, device: torch.device) -> None:
    """fn(t0, count, length, s0) for every group (s0 = index of its first segment); the second group
    runs on a side stream of `device`, joined before return, so the two launches share the GPU."""
    s0 = 0
    jobs = []
    for t0, count, length in groups:
        jobs.append((t0, count, length, s0))
        s0 += count
    if len(jobs) == 1:
        fn(*jobs[0])
        return
    cur = torch.cuda.current_stream(device)
    side = _SIDE.get(device.index)
    if side is None:
        side = _SIDE[device.index] = torch.cuda.Stream(device=device)
    side.wait_stream(cur)
    with torch.cuda.stream(cur):
        fn(*jobs[0])
    with torch.cuda.stream(side):
        for job in jobs[1:]:
            fn(*job)
    cur.wait_stream(side)


def segment_maps(q, k, v, alpha, beta, segments: Optional[int] = None, *, scale=None, chunk_size=CHUNK,
                 groups=None):
    """(A [S,H,K,K], B [S,H,K,V]) of the segments of a [1, T, H, D] span (pass 1): `segments`
    equal ones, or segment_groups for the device (or the given `groups`)."""
    T, H, K, V = q.shape[1], q.shape[2], q.shape[3], v.shape[3]
    if groups is None:
        groups = _resolve_groups(T, H, q.device, segments)
    S = sum(c for _, c, _ in groups)
    A = torch.empty((S, H, K, K), device=q.device, dtype=torch.float32)
    Bm = torch.empty((S, H, K, V), device=q.device, dtype=torch.float32)

    def run(t0, count, length, s0):
        view = lambda x: _group_view(x, t0, count, length)  # noqa: E731
        kernels.gdn2_span_transition(view(k), view(alpha), view(beta), transition=A[s0:s0 + count],
                                     chunk_size=chunk_size)
        kernels.gdn2_prefill(view(q), view(k), view(v), view(alpha), view(beta), scale=scale,
                             want_output=False, final_state=Bm[s0:s0 + count], chunk_size=chunk_size)

    _on_groups(groups, run, q.device)
    return A, Bm


def compose_maps(A: torch.Tensor, Bm: torch.Tensor):
    """The map of the whole span from its segment maps: (A_{S-1} ... A_0, fold of the B's)."""
    if A.is_cuda:
        _, Bt, At = kernels.gdn2_span_fold(A, Bm, None, want_composed=True)
        return At.unsqueeze(0), Bt.unsqueeze(0)
    At, Bt = A[0], Bm[0]
    for s in range(1, A.shape[0]):
        At = torch.matmul(A[s], At)
        Bt = torch.matmul(A[s], Bt) + Bm[s]
    return At.unsqueeze(0), Bt.unsqueeze(0)


def segment_starts(A: torch.Tensor, Bm: torch.Tensor, start: torch.Tensor) -> torch.Tensor:
    """Start states [S,H,K,V] of the S segments given the span's start state [1,H,K,V]."""
    if A.is_cuda:
        starts, _, _ = kernels.gdn2_span_fold(A, Bm, start[0], want_starts=True, want_end=False)
        return starts
    S = A.shape[0]
    out = torch.empty_like(Bm)
    s_cur = start[0]
    for s in range(S):
        out[s] = s_cur
        if s + 1 < S:
            s_cur = torch.matmul(A[s], s_cur) + Bm[s]
    return out


def segmented_prefill(q, k, v, alpha, beta, *, segments: Optional[int] = None, scale=None,
                      initial_state: Optional[torch.Tensor] = None, chunk_size: int = CHUNK,
                      maps=None, start: Optional[torch.Tensor] = None, starts: Optional[torch.Tensor] = None,
                      groups=None):
    """Prefill of one long sequence [1, T, H, D] on one GPU through time segmentation.

    Returns (out [1, T, H, V], final_state [1, H, K, V]).  Without ``maps`` this is one C-ABI call
    (kernels.gdn2_prefill_segmented: pass 1, fold and rescan in the library); ``maps`` reuses
    pass-1 results computed by the caller (``segment_maps`` with the same ``segments`` / ``groups``)
    and ``start`` overrides the span's start state (the multi-GPU driver, which has already
    computed the maps to hand them off); ``starts`` [S, H, K, V] are the segment start states when
    the caller has already folded them.
    """
    if q.shape[0] != 1:
        raise ValueError("segmented_prefill handles one sequence (batch 1)")
    T, H = q.shape[1], q.shape[2]
    if maps is None and segments is None and groups is None and chunk_size == CHUNK:
        # the library's own schedule (a lead segment beside the maps of the others)
        return kernels.gdn2_prefill_segmented(q, k, v, alpha, beta, segments=0, scale=scale,
                                              initial_state=start if start is not None else initial_state)
    if groups is None:
        groups = _resolve_groups(T, H, q.device, segments)
    S = 0 if groups is None else sum(c for _, c, _ in groups)
    if S <= 1:
        return kernels.gdn2_prefill(q, k, v, alpha, beta, scale=scale,
                                    initial_state=start if start is not None else initial_state,
                                    chunk_size=chunk_size)
    if maps is None:
        if len(groups) == 1:
            return kernels.gdn2_prefill_segmented(q, k, v, alpha, beta, segments=S, scale=scale,
                                                  initial_state=start if start is not None else initial_state)
        maps = segment_maps(q, k, v, alpha, beta, scale=scale, chunk_size=chunk_size, groups=groups)
    A, Bm = maps
    K, V = q.shape[3], v.shape[3]
    if start is None:
        start = initial_state if initial_state is not None else torch.zeros(
            (1, H, K, V), device=q.device, dtype=torch.float32)
    if starts is None:
        starts = segment_starts(A, Bm, start.to(torch.float32))
    out = torch.empty((1, T, H, V), device=q.device, dtype=q.dtype)
    fin = torch.empty((S, H, K, V), device=q.device, dtype=torch.float32)

    def run(t0, count, length, s0):
        view = lambda x: _group_view(x, t0, count, length)  # noqa: E731
        kernels.gdn2_prefill(view(q), view(k), view(v), view(alpha), view(beta), scale=scale,
                             initial_state=starts[s0:s0 + count], out=view(out),
                             final_state=fin[s0:s0 + count], chunk_size=chunk_size)

    _on_groups(groups, run, q.device)
    return out, fin[S - 1:S]


def time_sharded_prefill(q, k, v, alpha, beta, *, group=None, scale: Optional[float] = None,
                         initial_state: Optional[torch.Tensor] = None, chunk_size: int = CHUNK,
                         segments: Optional[int] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """Prefill of one rank's time span of a sequence sharded along time.

    q, k, v [1, T_span, H, D] and alpha, beta [1, T_span, H] are this rank's contiguous span (rank
    order = time order).  ``initial_state`` is the sequence's initial state (rank 0 only).  Returns
    this rank's outputs [1, T_span, H, V] and the state at the end of its span (on the last rank,
    the sequence's final state).
    """
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    if world == 1:
        return segmented_prefill(q, k, v, alpha, beta, segments=segments, scale=scale,
                                 initial_state=initial_state, chunk_size=chunk_size)
    T, H = q.shape[1], q.shape[2]
    groups = _resolve_groups(T, H, q.device, segments)
    if groups is None or sum(c for _, c, _ in groups) == 1:
        # unsegmented span: rank 0 scans from the initial state, the others hand off (A_g, B_g)
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
    maps = segment_maps(q, k, v, alpha, beta, scale=scale, chunk_size=chunk_size, groups=groups)
    K, V = q.shape[3], v.shape[3]
    starts = None
    if rank == 0:
        s0 = initial_state.to(torch.float32) if initial_state is not None else torch.zeros(
            (1, H, K, V), device=q.device, dtype=torch.float32)
        # the segment starts and the span's end state in one fold
        starts, end = rank0_fold(maps, s0)
        exchange_span_states(end.unsqueeze(0), None, rank, world, group)
        start = s0
    else:
        At, Bt = compose_maps(*maps)
        As, Bs = exchange_span_states(At, Bt, rank, world, group)
        start = fold_span_states(Bs[0], As, Bs, rank)
    return segmented_prefill(q, k, v, alpha, beta, scale=scale, chunk_size=chunk_size, groups=groups,
                             maps=maps, start=start, starts=starts)


def rank0_fold(maps, s0: torch.Tensor):
    """Segment starts [S,H,K,V] and end state [H,K,V] of the first rank's span from its start
    state s0 [1,H,K,V] (one fold kernel on CUDA tensors)."""
    A, Bm = maps
    if A.is_cuda:
        starts, end, _ = kernels.gdn2_span_fold(A, Bm, s0[0], want_starts=True, want_end=True)
        return starts, end
    starts = segment_starts(A, Bm, s0)
    return starts, torch.matmul(A[-1], starts[-1]) + Bm[-1]


class TimeShardedPrefillGraph:
    """``time_sharded_prefill`` of fixed inputs captured as one CUDA graph per rank.

    The step is many short launches (two map launches, the fold kernels, the packing copy, the
    ``all_gather``, the rescan) issued from Python, so a rank whose host falls behind holds every
    other rank at the collective.  Capturing the whole step (NCCL supports graph capture) replays
    it with no host work between launches.  The inputs are the tensors given here: write new
    values into them (``copy_``) and call ``replay()``; ``out`` and ``final_state`` are rewritten
    in place by every replay.  Every rank must construct, replay and ``release()`` the graph in
    the same order (the capture runs the collective twice during warm-up and once in the
    capture).  Call ``release()`` before ``destroy_process_group``.
    """

    def __init__(self, q, k, v, alpha, beta, *, group=None, scale: Optional[float] = None,
                 initial_state: Optional[torch.Tensor] = None, chunk_size: int = CHUNK,
                 segments: Optional[int] = None, warmup: int = 2):
        if not q.is_cuda:
            raise ValueError("TimeShardedPrefillGraph needs CUDA tensors")
        self._args = (q, k, v, alpha, beta)
        self._kw = dict(group=group, scale=scale, initial_state=initial_state, chunk_size=chunk_size,
                        segments=segments)
        dev = q.device
        cur = torch.cuda.current_stream(dev)
        side = torch.cuda.Stream(dev)
        side.wait_stream(cur)
        with torch.cuda.stream(side):
            for _ in range(max(1, warmup)):
                time_sharded_prefill(*self._args, **self._kw)
        cur.wait_stream(side)
        torch.cuda.synchronize(dev)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.out, self.final_state = time_sharded_prefill(*self._args, **self._kw)

    def replay(self) -> Tuple[torch.Tensor, torch.Tensor]:
        """One step on the current values of the inputs; returns (out, final_state)."""
        if self.graph is None:
            raise RuntimeError("TimeShardedPrefillGraph was released")
        self.graph.replay()
        return self.out, self.final_state

    def release(self) -> None:
        """Frees the graph (and the collective it holds)."""
        self.graph = None
