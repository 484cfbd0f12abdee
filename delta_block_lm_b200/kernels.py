"""Host mirror of the reference kernels crate's GDN-2 entry points, over torch CUDA tensors.

Each function validates like the reference (same conditions, messages adapted), allocates its
outputs like the reference's ops (which return fresh tensors, ``gdn_training.rs:391-393``), and
calls the C ABI of ``libdbl_gdn2.so`` on the current CUDA stream.  torch is only the plumbing
(device memory and streams); every kernel is this package's own CUDA code.

    gdn_training_scan  <- delta_kernels::gdn_training_scan  (crates/kernels/src/gdn_training_ops.rs:288-333)
    gdn_training_backward <- GdnTrainingOps::gdn_training_backward (gdn_training_ops.rs:95-127)
    gdn2_prologue      <- the GDN-2 gate and input producer of Mixer::forward_inner (crates/mixers/src/lib.rs:446-528)
    gdn2_scan          <- delta_kernels::gdn2_scan          (crates/kernels/src/ops.rs:251-276)
    gdn2_scan_backward <- Gdn2Ops::gdn2_backward            (ops.rs:106-160; kernels gdn2.rs:285-519)
    gdn2_prefill       <- scalar-gate chunked forward (the BASELINE prefill; chunk.rs:129-250 semantics)
    gdn2_prefill_host     the same from host buffers, copies and kernels pipelined over batch slices
    gdn2_span_transition  hand-off matrix for time-sharded prefill (no reference counterpart)
    gdn2_decode_step   <- the T = 1 continuation scan (crates/mixers/src/lib.rs:544-556), in place
"""
from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass
from typing import Optional

import torch

from . import _native as N


def _dtype_code(t: torch.Tensor) -> int:
    if t.dtype == torch.float32:
        return N.DBL_F32
    if t.dtype == torch.bfloat16:
        return N.DBL_BF16
    raise ValueError(f"unsupported dtype {t.dtype}: expected float32 or bfloat16")


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _require_cuda(*tensors: Optional[torch.Tensor]) -> torch.device:
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise ValueError("GDN-2 kernels require CUDA tensors; no CPU fallback")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError("GDN-2 inputs must share a device")
    if dev is None:
        raise ValueError("no tensor given")
    return dev


def _f32c(t: torch.Tensor) -> torch.Tensor:
    return t.to(torch.float32).contiguous()


@dataclass
class GdnTrainingOutput:
    """Mirror of delta_kernels::GdnTrainingOutput (gdn_training_ops.rs:276-282)."""

    output: torch.Tensor        # [B,T,H,V] f32
    final_state: torch.Tensor   # [B,H,K,V] f32
    scores: torch.Tensor        # [B,T,H,1] f32: |k| |edit| after decay


def gdn_training_scan(q, k, v, alpha, erase, write, valid, reset, initial, chunk_size: int
                      ) -> GdnTrainingOutput:
    """Fused GDN-2 forward with initial state, final state and physical scores.

    Shapes as the reference: q,k,alpha,erase [B,T,H,K]; v,write [B,T,H,V]; valid,reset [B,T]
    {0,1}; initial [B,H,K,V].  chunk_size 1..=16 (it bounds the reference's backward
    checkpoints; this forward-only build validates it and otherwise ignores it).
    """
    return _training_scan(q, k, v, alpha, erase, write, valid, reset, initial, chunk_size, False)[0]


def gdn_training_scan_saved(q, k, v, alpha, erase, write, valid, reset, initial, chunk_size: int):
    """gdn_training_scan that also returns the context its backward reads, as the reference's
    forward returns checkpoint and auxiliary tensors beside its outputs
    (gdn_training_ops.rs:201-224).  Returns (GdnTrainingOutput, context): context is a uint8 tensor,
    empty at shapes where the backward recomputes instead (chunk_size other than 16, wider keys or
    values, many sequence-heads); pass it to gdn_training_backward_saved with the same inputs."""
    return _training_scan(q, k, v, alpha, erase, write, valid, reset, initial, chunk_size, True)


def _training_scan(q, k, v, alpha, erase, write, valid, reset, initial, chunk_size, save):
    dev = _require_cuda(q, k, v, alpha, erase, write, valid, reset, initial)
    B, T, H, K = q.shape
    V = v.shape[3]
    if B == 0 or T == 0 or H == 0:
        raise ValueError("GDN-2 requires nonempty axes")
    for name, t, shape in (("k", k, (B, T, H, K)), ("v", v, (B, T, H, V)),
                           ("alpha", alpha, (B, T, H, K)), ("erase", erase, (B, T, H, K)),
                           ("write", write, (B, T, H, V)), ("valid", valid, (B, T)),
                           ("reset", reset, (B, T)), ("initial", initial, (B, H, K, V))):
        if tuple(t.shape) != shape:
            raise ValueError(f"{name} must have shape {list(shape)}, got {list(t.shape)}")
    if not 1 <= chunk_size <= 16:
        raise ValueError("GDN-2 checkpoint chunk must be 1..=16")
    dt = _dtype_code(q)
    if k.dtype != q.dtype or v.dtype != q.dtype:
        raise ValueError("q, k and v must share a dtype")
    with torch.cuda.device(dev):
        q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
        alpha, erase, write = _f32c(alpha), _f32c(erase), _f32c(write)
        valid, reset, initial = _f32c(valid), _f32c(reset), _f32c(initial)
        output = torch.empty((B, T, H, V), device=dev, dtype=torch.float32)
        final = torch.empty((B, H, K, V), device=dev, dtype=torch.float32)
        scores = torch.empty((B, T, H, 1), device=dev, dtype=torch.float32)
        a = N.TrainingScanArgs(B, T, H, K, V, dt, chunk_size, _ptr(q), _ptr(k), _ptr(v), _ptr(alpha),
                               _ptr(erase), _ptr(write), _ptr(valid), _ptr(reset), _ptr(initial),
                               _ptr(output), _ptr(final), _ptr(scores))
        ctx = None
        if save:
            need = N.lib().dbl_gdn_training_scan_context_bytes(B, T, H, K, V, chunk_size)
            ctx = torch.empty(need, device=dev, dtype=torch.uint8)
            N.check(N.lib().dbl_gdn_training_scan_save(ctypes.byref(a), _ptr(ctx) if need else None, need,
                                                       _stream(dev)))
        else:
            N.check(N.lib().dbl_gdn_training_scan(ctypes.byref(a), _stream(dev)))
    return GdnTrainingOutput(output, final, scores), ctx


@dataclass
class GdnTrainingGrads:
    """Gradients of gdn_training_scan's inputs, in the order the reference's backward returns them
    (gdn_training_ops.rs:95-127): q, k, v, alpha, erase, write, initial."""

    dq: torch.Tensor
    dk: torch.Tensor
    dv: torch.Tensor
    dalpha: torch.Tensor
    derase: torch.Tensor
    dwrite: torch.Tensor
    dinitial: torch.Tensor


def gdn_training_backward(q, k, v, alpha, erase, write, valid, reset, initial, grad_output,
                          grad_final_state=None, grad_scores=None, chunk_size: int = 16
                          ) -> GdnTrainingGrads:
    """Backward of gdn_training_scan for L = sum grad_output.output + sum grad_final_state.final_state
    + sum grad_scores.scores.  f32 as the reference's backward (K <= 64, V <= 256); the reference's
    packed upstream tensor is passed as its three parts; checkpoints are recomputed (chunk_size
    1..=16 is their spacing) instead of being read from the forward."""
    return _training_backward(q, k, v, alpha, erase, write, valid, reset, initial, grad_output, grad_final_state,
                              grad_scores, chunk_size, None)


def gdn_training_backward_saved(q, k, v, alpha, erase, write, valid, reset, initial, grad_output, context,
                                grad_final_state=None, grad_scores=None, chunk_size: int = 16
                                ) -> GdnTrainingGrads:
    """gdn_training_backward from the context gdn_training_scan_saved returned for the same inputs
    (the reference's backward consumes its forward's checkpoint and auxiliary tensors,
    gdn_training_ops.rs:87-112): the forward is not run again."""
    if context is None or not context.is_cuda or context.dtype != torch.uint8:
        raise ValueError("context must be the uint8 CUDA tensor gdn_training_scan_saved returned")
    return _training_backward(q, k, v, alpha, erase, write, valid, reset, initial, grad_output, grad_final_state,
                              grad_scores, chunk_size, context)


def _training_backward(q, k, v, alpha, erase, write, valid, reset, initial, grad_output, grad_final_state,
                       grad_scores, chunk_size, context):
    dev = _require_cuda(q, k, v, alpha, erase, write, valid, reset, initial, grad_output)
    B, T, H, K = q.shape
    V = v.shape[3]
    if B == 0 or T == 0 or H == 0:
        raise ValueError("GDN-2 requires nonempty axes")
    for name, t, shape in (("k", k, (B, T, H, K)), ("v", v, (B, T, H, V)),
                           ("alpha", alpha, (B, T, H, K)), ("erase", erase, (B, T, H, K)),
                           ("write", write, (B, T, H, V)), ("valid", valid, (B, T)),
                           ("reset", reset, (B, T)), ("initial", initial, (B, H, K, V)),
                           ("grad_output", grad_output, (B, T, H, V)),
                           ("grad_final_state", grad_final_state, (B, H, K, V)),
                           ("grad_scores", grad_scores, (B, T, H))):
        if t is not None and tuple(t.shape) != shape and not (name == "grad_scores" and tuple(t.shape) == (B, T, H, 1)):
            raise ValueError(f"{name} must have shape {list(shape)}, got {list(t.shape)}")
    if not 1 <= chunk_size <= 16:
        raise ValueError("GDN-2 checkpoint chunk must be 1..=16")
    lib = N.lib()
    with torch.cuda.device(dev):
        f = [_f32c(x) for x in (q, k, v, alpha, erase, write, valid, reset, initial, grad_output)]
        gf = None if grad_final_state is None else _f32c(grad_final_state)
        gs = None if grad_scores is None else _f32c(grad_scores)
        dq, dk, da, de = (torch.empty((B, T, H, K), device=dev, dtype=torch.float32) for _ in range(4))
        dv, dw = (torch.empty((B, T, H, V), device=dev, dtype=torch.float32) for _ in range(2))
        di = torch.empty((B, H, K, V), device=dev, dtype=torch.float32)
        need = lib.dbl_gdn_training_scan_backward_workspace_bytes(B, T, H, K, V, chunk_size)
        ws = torch.empty(max(need, 1), device=dev, dtype=torch.uint8)
        a = N.TrainingScanBackwardArgs(B, T, H, K, V, chunk_size, *(_ptr(x) for x in f[:9]), _ptr(f[9]),
                                       _ptr(gf), _ptr(gs), _ptr(dq), _ptr(dk), _ptr(dv), _ptr(da), _ptr(de),
                                       _ptr(dw), _ptr(di))
        if context is None:
            N.check(lib.dbl_gdn_training_scan_backward(ctypes.byref(a), _ptr(ws), need, _stream(dev)))
        else:
            N.check(lib.dbl_gdn_training_scan_backward_saved(ctypes.byref(a), _ptr(context) if context.numel() else None,
                                                             context.numel(), _ptr(ws), need, _stream(dev)))
    return GdnTrainingGrads(dq, dk, dv, da, de, dw, di)


def gdn2_prologue(proj_q, proj_k, proj_v, proj_decay, proj_erase, proj_write, conv_q, conv_k, conv_v,
                  decay_bias, decay_scale, valid, reset, heads: int, out_dtype=torch.float32):
    """GDN-2 mixer prologue (lib.rs:446-528): returns (q, k, v, alpha, erase, write) shaped for the
    scan -- q, k, alpha, erase [B,T,H,K], v, write [B,T,H,V]; q, k, v in ``out_dtype``, gates f32.
    Projections [B,T,H*K] / [B,T,H*V] (f32 or bf16); conv weights [W,H*K] / [W,H*V]; decay_bias
    [H*K] (or [H,K]); decay_scale [H]; valid, reset [B,T]."""
    dev = _require_cuda(proj_q, proj_k, proj_v, proj_decay, proj_erase, proj_write, conv_q, conv_k, conv_v,
                        decay_bias, decay_scale, valid, reset)
    B, T, HK = proj_q.shape
    HV = proj_v.shape[2]
    if HK % heads or HV % heads:
        raise ValueError("projection widths must be multiples of the head count")
    K, V = HK // heads, HV // heads
    W = conv_q.shape[0]
    for name, t, shape in (("proj_k", proj_k, (B, T, HK)), ("proj_decay", proj_decay, (B, T, HK)),
                           ("proj_erase", proj_erase, (B, T, HK)), ("proj_write", proj_write, (B, T, HV)),
                           ("conv_q", conv_q, (W, HK)), ("conv_k", conv_k, (W, HK)), ("conv_v", conv_v, (W, HV)),
                           ("valid", valid, (B, T)), ("reset", reset, (B, T))):
        if tuple(t.shape) != shape:
            raise ValueError(f"{name} must have shape {list(shape)}, got {list(t.shape)}")
    if decay_bias.numel() != HK or decay_scale.numel() != heads:
        raise ValueError("decay_bias needs H*K values and decay_scale H values")
    in_code = _dtype_code(proj_q)
    if any(x.dtype != proj_q.dtype for x in (proj_k, proj_v, proj_decay, proj_erase, proj_write)):
        raise ValueError("the six projections must share a dtype")
    out_code = N.DBL_BF16 if out_dtype == torch.bfloat16 else N.DBL_F32
    with torch.cuda.device(dev):
        pr = [x.contiguous() for x in (proj_q, proj_k, proj_v, proj_decay, proj_erase, proj_write)]
        fl = [_f32c(x) for x in (conv_q, conv_k, conv_v, decay_bias, decay_scale, valid, reset)]
        q, k = (torch.empty((B, T, heads, K), device=dev, dtype=out_dtype) for _ in range(2))
        v = torch.empty((B, T, heads, V), device=dev, dtype=out_dtype)
        alpha, erase = (torch.empty((B, T, heads, K), device=dev, dtype=torch.float32) for _ in range(2))
        write = torch.empty((B, T, heads, V), device=dev, dtype=torch.float32)
        a = N.Gdn2PrologueArgs(B, T, heads, K, V, W, in_code, out_code, *(_ptr(x) for x in pr), *(_ptr(x) for x in fl),
                               _ptr(q), _ptr(k), _ptr(v), _ptr(alpha), _ptr(erase), _ptr(write))
        N.check(N.lib().dbl_gdn2_prologue(ctypes.byref(a), _stream(dev)))
    return q, k, v, alpha, erase, write


def gdn2_scan(q, k, v, alpha, erase, write, doc_start, doc_end) -> torch.Tensor:
    """Output-only GDN-2 scan with inclusive document limits (ops.rs:251-276).

    Gates are cast to f32 like the reference (``ops.rs:261-264``).  Output in the q dtype.
    """
    dev = _require_cuda(q, k, v, alpha, erase, write, doc_start, doc_end)
    B, T, H, K = q.shape
    V = v.shape[3]
    if B == 0 or T == 0 or H == 0:
        raise ValueError("GDN-2 requires nonempty axes")
    for name, t, shape in (("k", k, (B, T, H, K)), ("v", v, (B, T, H, V)),
                           ("alpha", alpha, (B, T, H, K)), ("erase", erase, (B, T, H, K)),
                           ("write", write, (B, T, H, V)), ("doc_start", doc_start, (B, T)),
                           ("doc_end", doc_end, (B, T))):
        if tuple(t.shape) != shape:
            raise ValueError(f"{name} must have shape {list(shape)}, got {list(t.shape)}")
    dt = _dtype_code(q)
    with torch.cuda.device(dev):
        q, k, v = q.contiguous(), k.to(q.dtype).contiguous(), v.to(q.dtype).contiguous()
        alpha, erase, write = _f32c(alpha), _f32c(erase), _f32c(write)
        ds = doc_start.to(torch.int32).contiguous()
        de = doc_end.to(torch.int32).contiguous()
        out = torch.empty((B, T, H, V), device=dev, dtype=q.dtype)
        a = N.Gdn2ScanArgs(B, T, H, K, V, dt, _ptr(q), _ptr(k), _ptr(v), _ptr(alpha), _ptr(erase),
                           _ptr(write), _ptr(ds), _ptr(de), _ptr(out))
        N.check(N.lib().dbl_gdn2_scan(ctypes.byref(a), _stream(dev)))
    return out


def gdn2_scan_backward(q, k, v, alpha, erase, write, doc_start, doc_end, grad_output):
    """Backward of ``gdn2_scan`` (``Gdn2Ops::gdn2_backward``, crates/kernels/src/ops.rs:106-160;
    kernels gdn2.rs:285-519): returns (dq, dk, dv, dalpha, derase, dwrite), dq/dk/dv in the q dtype,
    the gate gradients f32.  The chunk states are recomputed; no forward checkpoint is needed."""
    dev = _require_cuda(q, k, v, alpha, erase, write, doc_start, doc_end, grad_output)
    B, T, H, K = q.shape
    V = v.shape[3]
    for name, t, shape in (("k", k, (B, T, H, K)), ("v", v, (B, T, H, V)), ("alpha", alpha, (B, T, H, K)),
                           ("erase", erase, (B, T, H, K)), ("write", write, (B, T, H, V)),
                           ("doc_start", doc_start, (B, T)), ("doc_end", doc_end, (B, T)),
                           ("grad_output", grad_output, (B, T, H, V))):
        if tuple(t.shape) != shape:
            raise ValueError(f"{name} must have shape {list(shape)}, got {list(t.shape)}")
    dt = _dtype_code(q)
    with torch.cuda.device(dev):
        q, k, v = q.contiguous(), k.to(q.dtype).contiguous(), v.to(q.dtype).contiguous()
        go = grad_output.to(q.dtype).contiguous()
        alpha, erase, write = _f32c(alpha), _f32c(erase), _f32c(write)
        ds, de = doc_start.to(torch.int32).contiguous(), doc_end.to(torch.int32).contiguous()
        dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
        da, dE, dw = torch.empty_like(alpha), torch.empty_like(erase), torch.empty_like(write)
        need = int(N.lib().dbl_gdn2_scan_backward_workspace_bytes(B, T, H, K, V, dt))
        ws = torch.empty(max(need, 1), device=dev, dtype=torch.uint8)
        a = N.Gdn2ScanBackwardArgs(B, T, H, K, V, dt, _ptr(q), _ptr(k), _ptr(v), _ptr(alpha), _ptr(erase),
                                   _ptr(write), _ptr(ds), _ptr(de), _ptr(go), _ptr(dq), _ptr(dk), _ptr(dv),
                                   _ptr(da), _ptr(dE), _ptr(dw))
        N.check(N.lib().dbl_gdn2_scan_backward(ctypes.byref(a), _ptr(ws), need, _stream(dev)))
    return dq, dk, dv, da, dE, dw


def _strides(t: torch.Tensor, n: int):
    s = (ctypes.c_int64 * n)()
    for i, x in enumerate(t.stride()):
        s[i] = x
    return s


def _prefill_args(q, k, v, alpha, beta, scale, valid, reset, initial_state, out, final_state,
                  chunk_size) -> N.PrefillArgs:
    B, T, H, K = q.shape
    V = v.shape[3] if v is not None else K
    a = N.PrefillArgs()
    a.batch, a.time, a.heads, a.key_dim, a.value_dim = B, T, H, K, V
    a.dtype = _dtype_code(q)
    a.chunk_size = chunk_size
    a.scale = scale
    a.q, a.k = _ptr(q), _ptr(k)
    a.q_stride, a.k_stride = _strides(q, 4), _strides(k, 4)
    if v is not None:
        a.v, a.v_stride = _ptr(v), _strides(v, 4)
    a.alpha, a.beta = _ptr(alpha), _ptr(beta)
    a.alpha_stride, a.beta_stride = _strides(alpha, 3), _strides(beta, 3)
    a.valid, a.reset = _ptr(valid), _ptr(reset)
    a.initial_state = _ptr(initial_state)
    if out is not None:
        a.out, a.out_stride = _ptr(out), _strides(out, 4)
    a.final_state = _ptr(final_state)
    return a


def _check_prefill_inputs(q, k, v, alpha, beta, valid, reset):
    B, T, H, K = q.shape
    if B == 0 or T == 0 or H == 0:
        raise ValueError("GDN-2 requires nonempty axes")
    if tuple(k.shape) != (B, T, H, K):
        raise ValueError(f"k must have shape {[B, T, H, K]}, got {list(k.shape)}")
    if v is not None and tuple(v.shape[:3]) != (B, T, H):
        raise ValueError(f"v must have shape [B,T,H,V] with B,T,H = {B},{T},{H}")
    for name, t in (("alpha", alpha), ("beta", beta)):
        if tuple(t.shape) != (B, T, H):
            raise ValueError(f"{name} must have shape {[B, T, H]}, got {list(t.shape)}")
        if t.dtype != torch.float32:
            raise ValueError(f"{name} must be float32 (recurrence gates never use low precision)")
    if (valid is None) != (reset is None):
        raise ValueError("valid and reset must be given together")
    for name, t in (("k", k), ("v", v)):
        if t is not None and t.dtype != q.dtype:
            raise ValueError(f"{name} must have the dtype of q")


def gdn2_prefill(q, k, v, alpha, beta, *, scale: Optional[float] = None, valid=None, reset=None,
                 initial_state=None, out=None, final_state=None, chunk_size: int = 64,
                 want_output: bool = True):
    """Chunked GDN-2 prefill with scalar gates (1, 4).

    S_t = alpha_t S_{t-1} (I - beta_t k k^T) + beta_t v k^T and o_t = S_t (scale q_t), in the
    reference's key-major state layout.  q,k [B,T,H,K]; v [B,T,H,V] (f32 or bf16; strided views
    with unit inner stride are taken as they are); alpha, beta [B,T,H] f32; valid/reset [B,T];
    initial_state [B,H,K,V] f32.  Returns (out [B,T,H,V] in the q dtype or None, final_state
    [B,H,K,V] f32).  ``final_state`` may be the initial state tensor (in-place update).
    """
    dev = _require_cuda(q, k, v, alpha, beta, valid, reset, initial_state, out, final_state)
    _check_prefill_inputs(q, k, v, alpha, beta, valid, reset)
    B, T, H, K = q.shape
    V = v.shape[3]
    if scale is None:
        scale = 1.0 / math.sqrt(K)
    with torch.cuda.device(dev):
        if valid is not None:
            valid, reset = _f32c(valid), _f32c(reset)
        if initial_state is not None:
            initial_state = _f32c(initial_state)
        if out is None and want_output:
            out = torch.empty((B, T, H, V), device=dev, dtype=q.dtype)
        if final_state is None:
            final_state = torch.empty((B, H, K, V), device=dev, dtype=torch.float32)
        a = _prefill_args(q, k, v, alpha, beta, scale, valid, reset, initial_state, out,
                          final_state, chunk_size)
        N.check(N.lib().dbl_gdn2_prefill(ctypes.byref(a), _stream(dev)))
    return out, final_state


_host_streams: dict = {}


def gdn2_prefill_host(q, k, v, alpha, beta, *, device=None, scale: Optional[float] = None, out=None,
                      final_state=None, pieces: int = 8):
    """``gdn2_prefill`` from host buffers: copies the inputs to ``device``, runs the prefill and
    copies the output and the final state back, pipelined over ``pieces`` slices of the batch on
    separate CUDA streams, so that one slice's kernel and read-back overlap the next slices'
    host-to-device copies (the sequences of a batch are independent).  q, k, v, alpha, beta are
    host tensors (pinned, for asynchronous copies); ``out`` [B,T,H,V] and ``final_state`` [B,H,K,V]
    are host tensors (allocated pinned when not given).  The work is ordered before later work on
    the device's current stream; the host results are complete once that stream is synchronised.
    Returns (out, final_state)."""
    if q.is_cuda:
        raise ValueError("gdn2_prefill_host takes host tensors; use gdn2_prefill for device tensors")
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    B, T, H, K = q.shape
    V = v.shape[3]
    pieces = max(1, min(int(pieces), B))
    if out is None:
        out = torch.empty((B, T, H, V), dtype=q.dtype, pin_memory=True)
    if final_state is None:
        final_state = torch.empty((B, H, K, V), dtype=torch.float32, pin_memory=True)
    key = (dev.index, pieces)
    if key not in _host_streams:
        with torch.cuda.device(dev):
            _host_streams[key] = [torch.cuda.Stream(dev) for _ in range(pieces)]
    streams = _host_streams[key]
    main = torch.cuda.current_stream(dev)
    start = torch.cuda.Event()
    start.record(main)
    with torch.cuda.device(dev):
        for i, st in enumerate(streams):
            lo, hi = B * i // pieces, B * (i + 1) // pieces
            if lo == hi:
                continue
            st.wait_event(start)
            with torch.cuda.stream(st):
                dq, dk, dv = (x[lo:hi].to(dev, non_blocking=True) for x in (q, k, v))
                da, db = (x[lo:hi].to(dev, non_blocking=True) for x in (alpha, beta))
                o, f = gdn2_prefill(dq, dk, dv, da, db, scale=scale)
                out[lo:hi].copy_(o, non_blocking=True)
                final_state[lo:hi].copy_(f, non_blocking=True)
                done = torch.cuda.Event()
                done.record(st)
            main.wait_event(done)
    return out, final_state


def gdn2_span_transition(k, alpha, beta, *, valid=None, reset=None, transition=None,
                         chunk_size: int = 64) -> torch.Tensor:
    """Per-(b,h) K x K matrix A of the span: S_end = A S_start + (scan of the span from zero).

    The hand-off object of time-sharded prefill.  k [B,T,H,K]; gates [B,T,H] f32.
    """
    dev = _require_cuda(k, alpha, beta, valid, reset, transition)
    _check_prefill_inputs(k, k, None, alpha, beta, valid, reset)
    B, T, H, K = k.shape
    with torch.cuda.device(dev):
        if valid is not None:
            valid, reset = _f32c(valid), _f32c(reset)
        if transition is None:
            transition = torch.empty((B, H, K, K), device=dev, dtype=torch.float32)
        a = _prefill_args(k, k, None, alpha, beta, 1.0, valid, reset, None, None, None, chunk_size)
        N.check(N.lib().dbl_gdn2_span_transition(ctypes.byref(a), _ptr(transition), _stream(dev)))
    return transition


def gdn2_span_fold(transition, offset=None, start=None, *, want_starts=False, want_end=True,
                   want_composed=False):
    """Fold of consecutive span maps: X_{s+1} = transition[s] X_s + offset[s], X_0 = start.

    transition [S,H,K,K], offset [S,H,K,V] (None = zeros), start [H,K,V] (None = zeros), f32.
    Returns (starts [S,H,K,V] or None, end [H,K,V] or None, composed [H,K,K] or None): the start
    state of every span, the state after the last span and the composed transition
    transition[S-1] ... transition[0]."""
    dev = _require_cuda(transition, offset, start)
    S, H, K, _ = transition.shape
    V = offset.shape[3] if offset is not None else (start.shape[2] if start is not None else K)
    with torch.cuda.device(dev):
        transition = _f32c(transition)
        offset = None if offset is None else _f32c(offset)
        start = None if start is None else _f32c(start).reshape(H, K, V)
        starts = torch.empty((S, H, K, V), device=dev, dtype=torch.float32) if want_starts else None
        end = torch.empty((H, K, V), device=dev, dtype=torch.float32) if want_end else None
        comp = torch.empty((H, K, K), device=dev, dtype=torch.float32) if want_composed else None
        N.check(N.lib().dbl_gdn2_span_fold(_ptr(transition), _ptr(offset), S, H, K, V, _ptr(start), _ptr(starts),
                                           _ptr(end), _ptr(comp), _stream(dev)))
    return starts, end, comp


def gdn2_prefill_segmented(q, k, v, alpha, beta, *, segments: int = 0, scale: Optional[float] = None,
                           valid=None, reset=None, initial_state=None, out=None, final_state=None):
    """``gdn2_prefill`` of ONE long sequence (batch 1) on one device by time segments (pass 1 the
    segment maps, a fold of their start states, pass 2 the rescan), in one C-ABI call
    (dbl_gdn2_prefill_segmented).  segments = 0 lets the library pick the schedule: a lead segment
    scanned from the initial state beside the maps of floor(SMs / H) - 1 equal segments, then one
    rescan of floor(SMs / H) segments (T a multiple of 64), else the largest power of two with
    segments x H <= the SM count.  Returns (out [1,T,H,V], final_state [1,H,K,V])."""
    dev = _require_cuda(q, k, v, alpha, beta, valid, reset, initial_state, out, final_state)
    _check_prefill_inputs(q, k, v, alpha, beta, valid, reset)
    B, T, H, K = q.shape
    V = v.shape[3]
    if B != 1:
        raise ValueError("gdn2_prefill_segmented handles one sequence (batch 1)")
    if scale is None:
        scale = 1.0 / math.sqrt(K)
    with torch.cuda.device(dev):
        if valid is not None:
            valid, reset = _f32c(valid), _f32c(reset)
        if initial_state is not None:
            initial_state = _f32c(initial_state)
        if out is None:
            out = torch.empty((B, T, H, V), device=dev, dtype=q.dtype)
        if final_state is None:
            final_state = torch.empty((B, H, K, V), device=dev, dtype=torch.float32)
        a = _prefill_args(q, k, v, alpha, beta, scale, valid, reset, initial_state, out, final_state, 64)
        L = N.lib()
        need = int(L.dbl_gdn2_prefill_segmented_workspace_bytes(ctypes.byref(a), segments))
        ws = torch.empty(max(need, 256), device=dev, dtype=torch.uint8)
        N.check(L.dbl_gdn2_prefill_segmented(ctypes.byref(a), segments, _ptr(ws), need, _stream(dev)))
    return out, final_state


def gdn2_prefill_time_sharded_devices(spans, *, segments: int = 0, scale: Optional[float] = None,
                                      initial_state=None):
    """ONE long sequence sharded along time over several devices of this process, through the
    C-ABI's multi-device entry point (dbl_gdn2_prefill_time_sharded): ``spans`` is a list of
    (q, k, v, alpha, beta) tuples, the consecutive time spans of the sequence, each on its own
    device (batch 1).  Each device runs on its current stream; the span maps cross devices by peer
    copies.  Returns ([out_g per span], final_state on the last span's device)."""
    n = len(spans)
    args, devs, streams, wss, sizes, outs, keep = [], [], [], [], [], [], []
    fin = None
    for g, (q, k, v, alpha, beta) in enumerate(spans):
        dev = _require_cuda(q, k, v, alpha, beta)
        _check_prefill_inputs(q, k, v, alpha, beta, None, None)
        _, T, H, K = q.shape
        V = v.shape[3]
        sc = 1.0 / math.sqrt(K) if scale is None else scale
        with torch.cuda.device(dev):
            out = torch.empty((1, T, H, V), device=dev, dtype=q.dtype)
            init = _f32c(initial_state) if (g == 0 and initial_state is not None) else None
            if g == n - 1:
                fin = torch.empty((1, H, K, V), device=dev, dtype=torch.float32)
            a = _prefill_args(q, k, v, alpha, beta, sc, None, None, init, out, fin if g == n - 1 else None, 64)
            need = int(N.lib().dbl_gdn2_prefill_time_sharded_workspace_bytes(ctypes.byref(a), n, segments))
            ws = torch.empty(max(need, 256), device=dev, dtype=torch.uint8)
            stream = torch.cuda.current_stream(dev)
        args.append(a)
        devs.append(dev.index)
        streams.append(stream.cuda_stream)
        wss.append(ws.data_ptr())
        sizes.append(need)
        outs.append(out)
        keep += [ws, init]
    arr = (N.PrefillArgs * n)(*args)
    N.check(N.lib().dbl_gdn2_prefill_time_sharded(
        arr, n, (ctypes.c_int * n)(*devs), (ctypes.c_void_p * n)(*streams), segments,
        (ctypes.c_void_p * n)(*wss), (ctypes.c_size_t * n)(*sizes)))
    # device g's stream reads the workspaces of devices 0 .. g-1 (peer copies): every device's
    # stream waits for every other one, so a workspace freed below is not reused before those reads
    done = []
    for q, *_rest in spans:
        with torch.cuda.device(q.device):
            e = torch.cuda.Event()
            e.record(torch.cuda.current_stream(q.device))
            done.append(e)
    for q, *_rest in spans:
        for e in done:
            torch.cuda.current_stream(q.device).wait_event(e)
    del keep
    return outs, fin


def gdn2_decode_step(q, k, v, alpha, beta, state, *, scale: Optional[float] = None, out=None):
    """One recurrent step for N sequences; ``state`` [N,H,K,V] f32 is updated IN PLACE.

    q,k [N,H,K]; v [N,H,V] (f32 or bf16); alpha, beta [N,H] f32.  Returns out [N,H,V].
    """
    dev = _require_cuda(q, k, v, alpha, beta, state, out)
    Nn, H, K = q.shape
    V = v.shape[2]
    if tuple(k.shape) != (Nn, H, K) or tuple(v.shape[:2]) != (Nn, H):
        raise ValueError("decode: q,k must be [N,H,K] and v [N,H,V]")
    if tuple(state.shape) != (Nn, H, K, V) or state.dtype != torch.float32 or not state.is_contiguous():
        raise ValueError("decode: state must be a contiguous float32 [N,H,K,V] tensor")
    for name, t in (("alpha", alpha), ("beta", beta)):
        if tuple(t.shape) != (Nn, H) or t.dtype != torch.float32:
            raise ValueError(f"decode: {name} must be float32 [N,H]")
    if scale is None:
        scale = 1.0 / math.sqrt(K)
    with torch.cuda.device(dev):
        alpha, beta = alpha.contiguous(), beta.contiguous()
        if out is None:
            out = torch.empty((Nn, H, V), device=dev, dtype=q.dtype)
        a = N.DecodeArgs()
        a.batch, a.heads, a.key_dim, a.value_dim = Nn, H, K, V
        a.dtype = _dtype_code(q)
        a.scale = scale
        a.q, a.k, a.v = _ptr(q), _ptr(k), _ptr(v)
        a.q_stride, a.k_stride, a.v_stride = _strides(q, 3), _strides(k, 3), _strides(v, 3)
        a.alpha, a.beta = _ptr(alpha), _ptr(beta)
        a.state = _ptr(state)
        a.out, a.out_stride = _ptr(out), _strides(out, 3)
        N.check(N.lib().dbl_gdn2_decode_step(ctypes.byref(a), _stream(dev)))
    return out
