"""CPU tests of the C ABI boundary: the library loads, exports every function the header declares,
its structures match the ctypes mirror byte for byte, and argument errors come back as status
codes (no CUDA call is made before validation, so these run without a GPU)."""
import ctypes
import os
import re
import subprocess

import pytest

from delta_block_lm_b200 import _native as N

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "dbl_gdn2.h")

STRUCTS = {
    "dbl_prefill_args": N.PrefillArgs,
    "dbl_decode_args": N.DecodeArgs,
    "dbl_training_scan_args": N.TrainingScanArgs,
    "dbl_training_scan_backward_args": N.TrainingScanBackwardArgs,
    "dbl_gdn2_prologue_args": N.Gdn2PrologueArgs,
    "dbl_gdn2_scan_args": N.Gdn2ScanArgs,
    "dbl_gdn2_scan_backward_args": N.Gdn2ScanBackwardArgs,
    "dbl_relay_merge_args": N.RelayMergeArgs,
    "dbl_relay_attention_args": N.RelayAttentionArgs,
}


def declared_functions():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?[a-z_]+\s*\*?\s*(dbl_[a-z0-9_]+)\s*\(", text, re.M)))


def test_every_declared_function_is_exported(native_lib):
    names = declared_functions()
    assert len(names) >= 10
    for name in names:
        assert hasattr(native_lib, name), name
    assert {n for n, _, _ in N.EXPORTS} == set(names)


def test_struct_layout_matches_header(tmp_path):
    lines = ['#include <stdio.h>', '#include <stddef.h>', f'#include "{HEADER}"', "int main(void) {"]
    for cname, py in STRUCTS.items():
        lines.append(f'printf("{cname} size %zu\\n", sizeof({cname}));')
        for field, _ in py._fields_:
            lines.append(f'printf("{cname} {field} %zu\\n", offsetof({cname}, {field}));')
    lines.append("return 0; }")
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.check_call(["gcc", "-std=c11", "-o", str(exe), str(src)])
    out = subprocess.check_output([str(exe)], text=True).split("\n")
    got = {}
    for line in out:
        if line:
            s, f, v = line.split()
            got[(s, f)] = int(v)
    for cname, py in STRUCTS.items():
        assert got[(cname, "size")] == ctypes.sizeof(py), cname
        for field, _ in py._fields_:
            assert got[(cname, field)] == getattr(py, field).offset, (cname, field)


def test_status_strings_and_version(native_lib):
    assert native_lib.dbl_status_string(0) == b"ok"
    assert native_lib.dbl_status_string(N.DBL_ERR_WORKSPACE).startswith(b"workspace")
    assert native_lib.dbl_status_string(99) == b"unknown status"
    assert native_lib.dbl_abi_version() >= 10100


def test_null_and_bad_arguments_return_status(native_lib):
    assert native_lib.dbl_gdn2_prefill(None, None) == N.DBL_ERR_INVALID_ARGUMENT
    assert b"null" in native_lib.dbl_last_error()
    a = N.PrefillArgs()
    a.batch, a.time, a.heads, a.key_dim, a.value_dim = 1, 0, 1, 64, 64
    assert native_lib.dbl_gdn2_prefill(ctypes.byref(a), None) == N.DBL_ERR_INVALID_ARGUMENT
    assert b"nonempty" in native_lib.dbl_last_error()
    a.time, a.chunk_size = 4, 16
    assert native_lib.dbl_gdn2_prefill(ctypes.byref(a), None) == N.DBL_ERR_UNSUPPORTED
    t = N.TrainingScanArgs(1, 4, 1, 32, 64, N.DBL_F32, 17)
    assert native_lib.dbl_gdn_training_scan(ctypes.byref(t), None) == N.DBL_ERR_INVALID_ARGUMENT
    assert b"1..=16" in native_lib.dbl_last_error()
    d = N.DecodeArgs()
    d.batch, d.heads, d.key_dim, d.value_dim = 1, 1, 96, 128
    assert native_lib.dbl_gdn2_decode_step(ctypes.byref(d), None) == N.DBL_ERR_UNSUPPORTED
    r = N.RelayMergeArgs(1, 1, 100, 4, 4, N.DBL_BF16, 0.1)
    assert native_lib.dbl_relay_merge_decode(ctypes.byref(r), None, 0, None) == N.DBL_ERR_UNSUPPORTED


def test_relay_workspace_size_and_check(native_lib):
    need = native_lib.dbl_relay_merge_workspace_bytes(64, 16, 128, 4096, 1024)
    # 64 * 16 rows x (2 * 64 prefix + 1 own partial, the f32 layout) x (128 + 2) floats + counters
    assert need >= 64 * 16 * 129 * 130 * 4
    assert native_lib.dbl_relay_merge_workspace_bytes(0, 16, 128, 4096, 1024) == 0
    r = N.RelayMergeArgs(64, 16, 128, 4096, 1024, N.DBL_BF16, 0.088, 256, 256, 256, 256, 256, None, 256)
    assert native_lib.dbl_relay_merge_decode(ctypes.byref(r), None, need, None) == N.DBL_ERR_WORKSPACE
    assert native_lib.dbl_relay_merge_decode(ctypes.byref(r), 256, need - 1, None) == N.DBL_ERR_WORKSPACE


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    monkeypatch.setattr(N, "LIB_PATH", str(tmp_path / "absent.so"))
    monkeypatch.setattr(N, "_lib", None)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        N.lib()


def test_training_backward_workspace_and_checks(native_lib):
    f = native_lib.dbl_gdn_training_scan_backward_workspace_bytes
    # token-sequential backward: checkpoints (B*H*ceil(T/C)) plus one chunk of replayed states
    # (B*H*C), K*V floats each
    assert f(2, 40, 3, 32, 64, 8) == (2 * 3 * 5 + 2 * 3 * 8) * 32 * 64 * 4
    assert f(2, 40, 3, 32, 200, 16) == (2 * 3 * 3 + 2 * 3 * 16) * 32 * 200 * 4
    # chunked backward (16-token checkpoints, K <= 64, V <= 128, T >= 32): the chunk-start
    # states, every token's edit and its gradient, and each chunk end's state gradient at least
    assert f(2, 40, 3, 32, 64, 16) >= (2 * 3 * 3 * 32 * 64 * 2 + 2 * 40 * 3 * 64 * 2) * 4
    assert f(2, 40, 3, 32, 17, 16) % 16 == 0
    assert f(2, 40, 3, 32, 64, 17) == 0 and f(0, 40, 3, 32, 64, 16) == 0
    a = N.TrainingScanBackwardArgs(1, 8, 1, 32, 64, 0)
    assert native_lib.dbl_gdn_training_scan_backward(ctypes.byref(a), None, 0, None) == N.DBL_ERR_INVALID_ARGUMENT
    ptrs = {n: 256 for n, _ in N.TrainingScanBackwardArgs._fields_[6:] if n not in
            ("initial_state", "grad_final_state", "grad_scores", "dinitial")}
    a = N.TrainingScanBackwardArgs(1, 8, 1, 96, 64, 8, **ptrs)
    assert native_lib.dbl_gdn_training_scan_backward(ctypes.byref(a), 256, 1 << 30, None) == N.DBL_ERR_UNSUPPORTED
    a = N.TrainingScanBackwardArgs(1, 8, 1, 32, 64, 8, **ptrs)
    assert native_lib.dbl_gdn_training_scan_backward(ctypes.byref(a), 256, 16, None) == N.DBL_ERR_WORKSPACE


def test_training_context_sizes_and_checks(native_lib):
    # the saved forward context exists only at the chunked backward's shapes (chunk 16, K <= 64,
    # V <= 128, T >= 32); elsewhere it is empty
    f = native_lib.dbl_gdn_training_scan_context_bytes
    n = f(2, 40, 3, 32, 64, 16)
    assert n > 0 and n % 16 == 0
    # at least the chunk-start states and every token's edit
    assert n >= (2 * 3 * 3 * 32 * 64 + 2 * 40 * 3 * 64) * 4
    assert f(2, 40, 3, 32, 64, 8) == 0 and f(2, 40, 3, 32, 200, 16) == 0 and f(2, 20, 3, 32, 64, 16) == 0
    assert f(64, 40, 16, 32, 64, 16) > 0 and f(2, 40, 3, 96, 64, 16) == 0 and f(0, 40, 3, 32, 64, 16) == 0
    # argument checks, before anything is launched
    ptrs = {nm: 256 for nm, _ in N.TrainingScanArgs._fields_[7:] if nm not in
            ("initial_state", "final_state", "scores")}
    a = N.TrainingScanArgs(2, 40, 3, 32, 64, N.DBL_F32, 16, **ptrs)
    assert native_lib.dbl_gdn_training_scan_save(ctypes.byref(a), None, 0, None) == N.DBL_ERR_WORKSPACE
    assert native_lib.dbl_gdn_training_scan_save(ctypes.byref(a), 256, n - 1, None) == N.DBL_ERR_WORKSPACE
    assert native_lib.dbl_gdn_training_scan_save(ctypes.byref(a), 260, n, None) == N.DBL_ERR_INVALID_ARGUMENT
    bptrs = {nm: 256 for nm, _ in N.TrainingScanBackwardArgs._fields_[6:] if nm not in
             ("initial_state", "grad_final_state", "grad_scores", "dinitial")}
    b = N.TrainingScanBackwardArgs(2, 40, 3, 32, 64, 16, **bptrs)
    ws = native_lib.dbl_gdn_training_scan_backward_workspace_bytes(2, 40, 3, 32, 64, 16)
    assert native_lib.dbl_gdn_training_scan_backward_saved(ctypes.byref(b), None, 0, 256, ws, None) == \
        N.DBL_ERR_WORKSPACE
    assert native_lib.dbl_gdn_training_scan_backward_saved(ctypes.byref(b), 260, n, 256, ws, None) == \
        N.DBL_ERR_INVALID_ARGUMENT
    assert native_lib.dbl_gdn_training_scan_backward_saved(ctypes.byref(b), 256, n - 16, 256, ws, None) == \
        N.DBL_ERR_WORKSPACE
