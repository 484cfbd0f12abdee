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
