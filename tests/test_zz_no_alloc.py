"""The no-allocation relay entry point (dbl_relay_merge_decode_noalloc), through the C ABI.

This variant exists for callers that cannot allocate device memory where they call the relay
merge: a host whose device memory belongs to its own pooling allocator, or a serving loop that
must not call cudaMalloc/cudaFree while it runs.  Its partials live in a fixed array inside the
library, so these tests check that (1) two calls in a row -- on different inputs, so a stale
array would show -- agree with the workspace entry point dbl_relay_merge_decode within the
tolerance of the other relay tests, in bf16 and f32, at head widths 128 and 64, and at a shape
whose partials reach the last 64 KB of the array, and (2) a call too large for the array is
refused without launching anything.  The file name sorts last so that a run stopping at the first failure has
already run every other test; it also passes when run alone in a fresh process.
"""
import ctypes

import numpy as np
import pytest
import torch

from delta_block_lm_b200 import _native as N
from fixtures import TOL_BF16, TOL_F32, rel_err

pytestmark = pytest.mark.gpu
N_SCRATCH = 16 << 20  # DBL_RELAY_NOALLOC_SCRATCH_BYTES


def _args(q, kp, vp, ko, vo, out, row_max, row_sum, scale):
    n, h, d = q.shape
    dt = N.DBL_BF16 if q.dtype == torch.bfloat16 else N.DBL_F32
    return N.RelayMergeArgs(n, h, d, kp.shape[1], ko.shape[2], dt, scale, q.data_ptr(),
                            kp.data_ptr(), vp.data_ptr(), ko.data_ptr(), vo.data_ptr(), None,
                            out.data_ptr(), row_max.data_ptr(), row_sum.data_ptr())


# (dtype, n_seq, heads, head_dim, prefix_len, own_cap): a small bf16 case, a small f32 case with
# head width 64, and an f32 case whose partials fill the array to within 24 KB of its end
CASES = [(torch.bfloat16, 16, 4, 128, 1024, 700), (torch.float32, 8, 4, 64, 512, 300),
         (torch.float32, 61, 16, 64, 2048, 512)]


@pytest.mark.parametrize("dtype,n,h,d,lp,lo", CASES)
def test_noalloc_matches_workspace_entry_two_calls(cuda, native_lib, dtype, n, h, d, lp, lo):
    scale = 1.0 / np.sqrt(d)
    stream = torch.cuda.current_stream(cuda).cuda_stream
    need = native_lib.dbl_relay_merge_workspace_bytes(n, h, d, lp, lo)
    ws = torch.empty(need, device=cuda, dtype=torch.uint8)
    tol = TOL_BF16 if dtype == torch.bfloat16 else TOL_F32
    g = torch.Generator(device=cuda)
    for call in range(2):
        g.manual_seed(100 + call)
        mk = lambda *s: torch.randn(s, device=cuda, generator=g).to(dtype)  # noqa: E731
        q, kp, vp, ko, vo = mk(n, h, d), mk(h, lp, d), mk(h, lp, d), mk(n, h, lo, d), mk(n, h, lo, d)
        outs = []
        for noalloc in (False, True):
            out = torch.empty((n, h, d), device=cuda, dtype=dtype)
            rmax = torch.empty((n, h), device=cuda, dtype=torch.float32)
            rsum = torch.empty((n, h), device=cuda, dtype=torch.float32)
            a = _args(q, kp, vp, ko, vo, out, rmax, rsum, scale)
            if noalloc:
                own = native_lib.dbl_relay_merge_call_workspace_bytes(ctypes.byref(a))
                assert 0 < own <= N_SCRATCH
                if (n, lp) == (61, 2048):
                    assert own > N_SCRATCH - (64 << 10)  # the end of the array is written
                rc = native_lib.dbl_relay_merge_decode_noalloc(ctypes.byref(a), stream)
            else:
                rc = native_lib.dbl_relay_merge_decode(ctypes.byref(a), ws.data_ptr(), need, stream)
            assert rc == N.DBL_OK, native_lib.dbl_last_error()
            torch.cuda.synchronize()
            outs.append((out.float().cpu().numpy(), rmax.cpu().numpy(), rsum.cpu().numpy()))
        (o0, m0, s0), (o1, m1, s1) = outs
        assert rel_err(o1, o0) < tol, call
        assert rel_err(m1, m0) < tol and rel_err(s1, s0) < tol, call


def test_noalloc_refuses_calls_beyond_its_array(cuda, native_lib):
    # f32, 2 x 64 prefix partials per row: about 69 MB of partials, beyond the 16 MiB array
    n, h, d, lp, lo = 64, 16, 128, 4096, 1024
    dummy = torch.empty(16, device=cuda, dtype=torch.float32)
    p = dummy.data_ptr()
    a = N.RelayMergeArgs(n, h, d, lp, lo, N.DBL_F32, 0.1, p, p, p, p, p, None, p, None, None)
    rc = native_lib.dbl_relay_merge_decode_noalloc(ctypes.byref(a), None)
    assert rc == N.DBL_ERR_WORKSPACE
    assert b"fixed" in native_lib.dbl_last_error()
