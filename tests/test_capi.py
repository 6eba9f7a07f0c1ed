"""CPU tests of the C ABI: the library loads, exports every function that
include/cra.h declares, and its host-only helpers / argument validation
behave (no kernel is launched here)."""
import ctypes
import os
import re

import pytest

from oracle import cra_oracle as O

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "cra.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(cra_\w+)\s*\(", src)))


@pytest.fixture(scope="module")
def L():
    from cron_root_attention import _lib
    return _lib.lib()


def test_header_declares_expected_api():
    names = declared_functions()
    for n in ("cra_relay_build", "cra_fwd", "cra_bwd", "cra_bwd_workspace_bytes", "cra_window"):
        assert n in names


def test_library_exports_every_declared_symbol(L):
    from cron_root_attention import _lib
    for n in declared_functions():
        assert hasattr(L, n), n
        assert n in _lib.EXPORTED, f"{n} has no ctypes signature"


def test_window_matches_oracle(L):
    for S in list(range(1, 3000, 7)) + [65535, 65536, 65537, 262144, 524288, 10**9]:
        assert L.cra_window(S) == O.window(S), S


def test_relay_threshold_and_rows(L):
    assert L.cra_relay_active(2048) == 0 and L.cra_relay_active(2049) == 1
    for S in (1, 300, 2049, 65536, 524288):
        W = O.window(S)
        NB = (S + W - 1) // W
        assert L.cra_global_rows(S, 0, 2) == NB
        assert L.cra_global_rows(S, 1, 2) == 3 * NB
        assert L.cra_global_rows(S, 1, 4) == 5 * NB


def test_status_strings(L):
    for s in range(7):
        assert len(L.cra_status_string(s)) > 0
    assert L.cra_version() >= 100


def test_workspace_positive_and_monotone(L):
    a = L.cra_bwd_workspace_bytes(1, 16, 16, 65536, 128, 1, 2)
    b = L.cra_bwd_workspace_bytes(2, 16, 16, 65536, 128, 1, 2)
    assert a > 0 and b > a
    assert L.cra_bwd_workspace_bytes(1, 1, 1, 1, 96, 0, 2) == 0  # unsupported head_dim


def _st(*s):
    return (ctypes.c_int64 * 3)(*s)


def test_validation_errors_without_gpu(L):
    p = 0x100000
    st = _st(2 * 300 * 64, 300 * 64, 64)
    args = dict(B=1, H=2, Hkv=2, S=300, D=64)

    def fwd(q=p, D=64, H=2, Hkv=2, qs=st, scale=0.125):
        return L.cra_fwd(q, p, p, p, p, qs, st, st, 1, H, Hkv, 300, D, 0, 0, 2, ctypes.c_float(scale), p, st, p,
                         None, None)

    # rejected before any device work, with a detail message
    assert fwd(D=96) == 2
    assert b"head_dim" in L.cra_last_error_message()
    assert fwd(q=p + 2) == 3                      # misaligned base
    assert fwd(qs=_st(1, 300 * 64, 63)) == 3      # seq stride not a multiple of 8
    assert fwd(H=3, Hkv=2) == 1                   # heads % kv_heads
    assert fwd(scale=-1.0) == 1
    assert L.cra_fwd(None, p, p, p, p, st, st, st, 1, 2, 2, 300, 64, 0, 0, 2, ctypes.c_float(0.1), p, st, p,
                     None, None) == 1
    ws = L.cra_bwd_workspace_bytes(1, 2, 2, 300, 64, 0, 2)
    r = L.cra_bwd(p, p, p, p, p, p, p, p, p, st, st, st, st, st, 1, 2, 2, 300, 64, 0, 0, 2, ctypes.c_float(0.125),
                  None, p, p, p, st, st, st, None, p, ws - 1, None, None)
    assert r == 4 and b"workspace" in L.cra_last_error_message()


def test_wait_probe_library_loads():
    """The test-only bounded-wait probe library is built beside libcra and
    exports its one entry point (run on the GPU by test_wait_timeout_gpu)."""
    from test_wait_timeout_gpu import PROBE
    h = ctypes.CDLL(PROBE)
    assert hasattr(h, "cra_test_wait_timeout")


def test_varlen_plan_sizes(L):
    """Packed global rows and blocks of a varlen batch: each document with its
    own W = ceil(sqrt(len)) and relay switch (len > 2048)."""
    cu = (ctypes.c_int64 * 4)(0, 1000, 3100, 5000)
    exp_rows, exp_blocks = 0, 0
    for n in (1000, 2100, 1900):
        W = O.window(n)
        nb = (n + W - 1) // W
        exp_rows += nb * (3 if n > 2048 else 1)
        exp_blocks += nb
    assert L.cra_varlen_global_rows(cu, 3, 2) == exp_rows
    assert L.cra_varlen_blocks(cu, 3) == exp_blocks
    assert L.cra_varlen_table_bytes(3) == 3 * 32
    bad = (ctypes.c_int64 * 3)(0, 10, 10)
    assert L.cra_varlen_global_rows(bad, 2, 2) == -1
