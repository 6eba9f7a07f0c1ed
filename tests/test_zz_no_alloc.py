"""cra_bwd_noalloc: the backward for callers that cannot allocate device
memory (for example a plug-in whose host framework owns every allocation).
Called through the C ABI, its results must match cra_bwd with a
caller-provided workspace, on two calls in a row (the second call reuses the
library's fixed scratch left over from the first).  Collected last on
purpose; it also runs alone in a fresh process."""
import ctypes

import pytest
import torch

from parity import GRAD_REL_L2, inputs, rel_l2

pytestmark = pytest.mark.gpu


def _forward(L, _lib, q, k, v, dev):
    B, H, S, D = q.shape
    W = L.cra_window(S)
    NB = (S + W - 1) // W
    NG = L.cra_global_rows(S, 1, 2)
    gk = torch.empty(B, H, NG, D, device=dev, dtype=q.dtype)
    gv = torch.empty_like(gk)
    gsrc = torch.empty(B, H, NB, 2, device=dev, dtype=torch.int32)
    o = torch.empty_like(q)
    lse = torch.empty(B, H, S, device=dev, dtype=torch.float32)
    st = _lib.strides3
    s = torch.cuda.current_stream(dev).cuda_stream
    _lib.check(L.cra_relay_build(k.data_ptr(), v.data_ptr(), st(k), st(v), B, H, S, D, 1, 1, 2, None,
                                 gk.data_ptr(), gv.data_ptr(), gsrc.data_ptr(), s), "relay")
    _lib.check(L.cra_fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), gk.data_ptr(), gv.data_ptr(), st(q), st(k),
                         st(v), B, H, H, S, D, 1, 1, 2, ctypes.c_float(D ** -0.5), o.data_ptr(), st(o),
                         lse.data_ptr(), None, s), "fwd")
    return o, lse, gk, gv, gsrc


def _bwd_args(_lib, q, k, v, o, do, lse, gk, gv, gsrc, dq, dk, dv):
    B, H, S, D = q.shape
    st = _lib.strides3
    head = (q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), do.data_ptr(), lse.data_ptr(),
            gk.data_ptr(), gv.data_ptr(), gsrc.data_ptr(), st(q), st(k), st(v), st(o), st(do),
            B, H, H, S, D, 1, 1, 2, ctypes.c_float(D ** -0.5), None,
            dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), st(dq), st(dk), st(dv), None)
    return head


def test_noalloc_backward_matches_workspace_backward(cuda_device):
    from cron_root_attention import _lib
    L = _lib.lib()
    dev = cuda_device
    s = torch.cuda.current_stream(dev).cuda_stream
    for seed, S in ((40, 4100), (41, 3001)):  # two calls in a row, different sizes
        q, k, v, do = (t.to(dev) for t in inputs(1, 4, 4, S, 128, torch.bfloat16, seed, with_do=True))
        o, lse, gk, gv, gsrc = _forward(L, _lib, q, k, v, dev)
        ref = [torch.empty_like(t) for t in (q, k, v)]
        ws_bytes = L.cra_bwd_workspace_bytes(1, 4, 4, S, 128, 1, 2)
        assert 0 < ws_bytes <= 32 << 20
        ws = torch.empty(ws_bytes, device=dev, dtype=torch.uint8)
        _lib.check(L.cra_bwd(*_bwd_args(_lib, q, k, v, o, do, lse, gk, gv, gsrc, *ref), ws.data_ptr(), ws_bytes,
                             None, s), "cra_bwd")
        out = [torch.empty_like(t) for t in (q, k, v)]
        _lib.check(L.cra_bwd_noalloc(*_bwd_args(_lib, q, k, v, o, do, lse, gk, gv, gsrc, *out), None, s),
                   "cra_bwd_noalloc")
        torch.cuda.synchronize(dev)
        for a, b in zip(out, ref):
            assert rel_l2(a, b) <= GRAD_REL_L2
            assert torch.equal(a, b)  # same kernels, fixed summation order


def test_noalloc_rejects_sizes_beyond_its_scratch(cuda_device):
    from cron_root_attention import _lib
    L = _lib.lib()
    B, H, S, D = 1, 16, 65536, 128
    assert L.cra_bwd_workspace_bytes(B, H, H, S, D, 1, 2) > 32 << 20
    p = 0x100000
    st = (ctypes.c_int64 * 3)(H * S * D, S * D, D)
    r = L.cra_bwd_noalloc(p, p, p, p, p, p, p, p, p, st, st, st, st, st, B, H, H, S, D, 1, 1, 2,
                          ctypes.c_float(D ** -0.5), None, p, p, p, st, st, st, None, None, None)
    assert r == 4  # CRA_ERR_WORKSPACE
