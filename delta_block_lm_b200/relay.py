"""Host mirror of relay attention (decode case) over torch CUDA tensors.

``relay_merge_decode`` replaces, for the split shared-prefix / own-segment layout, the forward of
``RelayAttentionKernelOps::relay_attention_forward`` and its host
``run_relay_windowed_attention`` (reuse/crates/dre-attention/src/relay_attention_kernel.rs:14-20,
:311-340): it returns the output and the f32 ``[row maximum, sum(exp(score - maximum))]``
statistics per query, in the reference's convention.
"""
from __future__ import annotations

import ctypes
import math
from typing import Optional

import torch

from . import _native as N
from .kernels import _dtype_code, _ptr, _require_cuda, _stream


def relay_workspace_bytes(n_seq: int, heads: int, head_dim: int, prefix_len: int, own_cap: int) -> int:
    return int(N.lib().dbl_relay_merge_workspace_bytes(n_seq, heads, head_dim, prefix_len, own_cap))


def relay_merge_decode(q, prefix_k, prefix_v, own_k, own_v, *, scale: Optional[float] = None,
                       own_len=None, out=None, workspace: Optional[torch.Tensor] = None,
                       return_stats: bool = True):
    """One query per (sequence, head) over [shared prefix ; own segment], LSE-merged in one kernel.

    q [N,H,D]; prefix_k, prefix_v [H,Lp,D]; own_k, own_v [N,H,Lo,D]; own_len int [N] (ragged
    own segments) or None.  Returns (o [N,H,D], row_max [N,H], row_sum [N,H]).
    """
    dev = _require_cuda(q, prefix_k, prefix_v, own_k, own_v, own_len, out, workspace)
    Nn, H, D = q.shape
    Lp = prefix_k.shape[1]
    Lo = own_k.shape[2]
    if tuple(prefix_k.shape) != (H, Lp, D) or tuple(prefix_v.shape) != (H, Lp, D):
        raise ValueError("relay: prefix_k and prefix_v must be [H,Lp,D]")
    if tuple(own_k.shape) != (Nn, H, Lo, D) or tuple(own_v.shape) != (Nn, H, Lo, D):
        raise ValueError("relay: own_k and own_v must be [N,H,Lo,D]")
    for name, t in (("prefix_k", prefix_k), ("prefix_v", prefix_v), ("own_k", own_k), ("own_v", own_v)):
        if t.dtype != q.dtype:
            raise ValueError(f"relay: {name} must have the dtype of q")
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    with torch.cuda.device(dev):
        q, prefix_k, prefix_v = q.contiguous(), prefix_k.contiguous(), prefix_v.contiguous()
        own_k, own_v = own_k.contiguous(), own_v.contiguous()
        if own_len is not None:
            own_len = own_len.to(torch.int32).contiguous()
        if out is None:
            out = torch.empty((Nn, H, D), device=dev, dtype=q.dtype)
        row_max = torch.empty((Nn, H), device=dev, dtype=torch.float32) if return_stats else None
        row_sum = torch.empty((Nn, H), device=dev, dtype=torch.float32) if return_stats else None
        need = relay_workspace_bytes(Nn, H, D, Lp, Lo)
        if workspace is None:
            workspace = torch.empty(need, device=dev, dtype=torch.uint8)
        a = N.RelayMergeArgs(Nn, H, D, Lp, Lo, _dtype_code(q), scale, _ptr(q), _ptr(prefix_k),
                             _ptr(prefix_v), _ptr(own_k), _ptr(own_v), _ptr(own_len), _ptr(out),
                             _ptr(row_max), _ptr(row_sum))
        N.check(N.lib().dbl_relay_merge_decode(ctypes.byref(a), _ptr(workspace),
                                               workspace.numel() * workspace.element_size(),
                                               _stream(dev)))
    return out, row_max, row_sum


def relay_attention_forward(q, k, v, relay_k, relay_v, doc_id, doc_start, doc_end, *, out=None,
                            normalization=None):
    """Reference-layout relay attention (``relay_attention_forward`` / ``run_relay_windowed_attention``,
    reuse/crates/dre-attention/src/relay_attention_kernel.rs:14-20, :38-130, :311-340).

    q, k, v [B,H,T,64] and relay_k, relay_v [documents,H,16,64], f32 or bf16; doc_id, doc_start,
    doc_end [B,T] integer (inclusive limits; doc_end < doc_start marks padding).  Query t attends to
    the keys of [t - 128, t + 128] inside its document and to its document's 16 relay slots, with
    scores q.k / 8.  Returns (o [B,H,T,64] in the input dtype, normalization [B,H,T,2] f32 =
    (row maximum, sum of exp(score - maximum))); padding rows give o = 0 and (0, 1).
    """
    dev = _require_cuda(q, k, v, relay_k, relay_v, doc_id, doc_start, doc_end, out, normalization)
    B, H, T, D = q.shape
    if D != 64:
        raise ValueError("relay attention: head width must be 64")
    for name, t in (("k", k), ("v", v)):
        if tuple(t.shape) != (B, H, T, D):
            raise ValueError(f"relay attention: {name} must be [B,H,T,64], got {list(t.shape)}")
    nd = relay_k.shape[0]
    for name, t in (("relay_k", relay_k), ("relay_v", relay_v)):
        if tuple(t.shape) != (nd, H, 16, D):
            raise ValueError(f"relay attention: {name} must be [documents,H,16,64], got {list(t.shape)}")
    for name, t in (("doc_id", doc_id), ("doc_start", doc_start), ("doc_end", doc_end)):
        if tuple(t.shape) != (B, T):
            raise ValueError(f"relay attention: {name} must be [B,T], got {list(t.shape)}")
    for name, t in (("k", k), ("v", v), ("relay_k", relay_k), ("relay_v", relay_v)):
        if t.dtype != q.dtype:
            raise ValueError(f"relay attention: {name} must have the dtype of q")
    with torch.cuda.device(dev):
        q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
        relay_k, relay_v = relay_k.contiguous(), relay_v.contiguous()
        di, ds, de = (x.to(torch.int32).contiguous() for x in (doc_id, doc_start, doc_end))
        if out is None:
            out = torch.empty((B, H, T, D), device=dev, dtype=q.dtype)
        if normalization is None:
            normalization = torch.empty((B, H, T, 2), device=dev, dtype=torch.float32)
        a = N.RelayAttentionArgs(B, H, T, D, nd, _dtype_code(q), _ptr(q), _ptr(k), _ptr(v), _ptr(relay_k),
                                 _ptr(relay_v), _ptr(di), _ptr(ds), _ptr(de), _ptr(out), _ptr(normalization))
        N.check(N.lib().dbl_relay_attention_forward(ctypes.byref(a), _stream(dev)))
    return out, normalization
