"""Forward parity of the CUDA path (libcra through the public API and the C
ABI) against the CPU oracle and the reference's golden vectors."""
import ctypes
import glob
import os

import numpy as np
import pytest
import torch

from oracle import cra_oracle as O
from parity import fwd_check, inputs

pytestmark = pytest.mark.gpu

GOLDEN = sorted(glob.glob(os.path.join(os.path.dirname(__file__), "golden", "*.npz")))


def _cra():
    import cron_root_attention as cra
    return cra


def _run(q, k, v, dev, **kw):
    cra = _cra()
    o = cra.cron_root_attention(q.to(dev), k.to(dev), v.to(dev), **kw)
    torch.cuda.synchronize(dev)
    assert cra.check_device_errors(dev) == 0
    return o


@pytest.mark.parametrize("path", GOLDEN, ids=[os.path.basename(p) for p in GOLDEN])
def test_golden_vectors(path, cuda_device):
    from test_oracle import load_golden
    q, k, v, out, use_relay = load_golden(path)
    o = _run(q, k, v, cuda_device)
    r = fwd_check(o, out, q.dtype)
    assert r["ok"], r


CASES = [
    # B, H, S, D, dtype, seed, sigma
    (1, 2, 1, 64, torch.float16, 0, 1.0),
    (1, 2, 2, 64, torch.float16, 0, 1.0),
    (1, 1, 17, 128, torch.bfloat16, 1, 1.0),
    (1, 2, 128, 64, torch.float16, 2, 1.0),
    (1, 2, 129, 128, torch.float16, 3, 1.0),
    (1, 1, 255, 64, torch.bfloat16, 4, 1.0),
    (2, 2, 2048, 64, torch.float16, 5, 1.0),
    (1, 2, 2049, 128, torch.bfloat16, 6, 1.0),
    (1, 1, 3001, 64, torch.float16, 7, 1.0),
    (1, 2, 4096, 128, torch.bfloat16, 8, 1.0),
    (2, 2, 5000, 128, torch.float16, 9, 0.5),
]


@pytest.mark.parametrize("B,H,S,D,dt,seed,sigma", CASES)
def test_forward_vs_oracle(B, H, S, D, dt, seed, sigma, cuda_device):
    q, k, v = inputs(B, H, H, S, D, dt, seed, sigma)
    o = _run(q, k, v, cuda_device)
    ref, _ = O.forward(q, k, v)
    r = fwd_check(o, ref, dt, v_rms=sigma)
    assert r["ok"], r


def test_northstar_forward_every_row(cuda_device):
    """North-star shape (B1 H16 D128 S65536 bf16): two whole heads checked
    row by row against the oracle, three calls in a row (a race that corrupts
    one query tile now and then would show here)."""
    q, k, v = inputs(1, 16, 16, 65536, 128, torch.bfloat16, 2)
    for _ in range(3):
        o = _run(q, k, v, cuda_device)
        for h in (0, 11):
            ref, _ = O.forward(q[:, h:h + 1], k[:, h:h + 1], v[:, h:h + 1])
            r = fwd_check(o[:, h:h + 1], ref, torch.bfloat16)
            assert r["ok"], r


def test_config2_full_size(cuda_device):
    """B1 H12 D64 S16384 fp16, N(0,1)*0.5, seed 1."""
    q, k, v = inputs(1, 12, 12, 16384, 64, torch.float16, 1, 0.5)
    o = _run(q, k, v, cuda_device)
    ref, _ = O.forward(q, k, v)
    r = fwd_check(o, ref, torch.float16)
    assert r["ok"], r


def _device_inputs(B, H, S, D, dt, seed, sigma, dev):
    """Seeded inputs drawn on the device (q, k, v in that order, N(0,1) * sigma,
    cast to dt): the BASELINE shapes at full size are too large to draw on the
    host in reasonable time."""
    g = torch.Generator(device=dev).manual_seed(seed)
    return tuple((torch.randn(B, H, S, D, generator=g, device=dev) * sigma).to(dt) for _ in range(3))


def test_config4_full_size(cuda_device):
    """BASELINE config 4 at full size on one GPU: B1 H32 D128 S262144 fp16,
    N(0,1) * 0.5, seed 3 (device generator).  Two whole heads checked row by
    row against the oracle."""
    dev = cuda_device
    q, k, v = _device_inputs(1, 32, 262144, 128, torch.float16, 3, 0.5, dev)
    o = _cra().cron_root_attention(q, k, v)
    torch.cuda.synchronize(dev)
    assert _cra().check_device_errors(dev) == 0
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    for h in (0, 21):
        sl = lambda t: t[:, h:h + 1].cpu()
        ref, _ = O.forward(sl(q), sl(k), sl(v))
        r = fwd_check(sl(o), ref, torch.float16, v_rms=0.5)
        assert r["ok"], (h, r)


@pytest.mark.parametrize("top_k", [1, 3, 4])
def test_relay_top_k(top_k, cuda_device):
    q, k, v = inputs(1, 2, 2, 2600, 64, torch.float16, 20 + top_k)
    o = _run(q, k, v, cuda_device, relay_top_k=top_k)
    ref, _ = O.forward(q, k, v, top_k=top_k)
    _r = fwd_check(o, ref, torch.float16)
    assert _r["ok"], _r


def test_relay_log_scale_forward(cuda_device):
    q, k, v = inputs(1, 2, 2, 2600, 128, torch.float16, 30)
    a = torch.tensor([0.3, -0.5])
    o = _run(q, k, v, cuda_device, relay_log_scale=a.to(cuda_device))
    ref, _ = O.forward(q, k, v, relay_log_scale=a, relay_dtype=torch.float16)
    _r = fwd_check(o, ref, torch.float16)
    assert _r["ok"], _r


def test_gqa_forward(cuda_device):
    q, k, v = inputs(1, 4, 2, 2500, 64, torch.bfloat16, 31)
    o = _run(q, k, v, cuda_device, kv_groups=2)
    ref, _ = O.forward(q, k, v, kv_groups=2)
    _r = fwd_check(o, ref, torch.bfloat16)
    assert _r["ok"], _r


def test_non_contiguous_inputs(cuda_device):
    """[B, S, H, D] storage viewed as [B, H, S, D] (what the modules pass)."""
    g = torch.Generator().manual_seed(32)
    x = torch.randn(3, 1, 2300, 2, 64, generator=g).half()
    q, k, v = (x[i].transpose(1, 2) for i in range(3))
    o = _run(q, k, v, cuda_device)
    ref, _ = O.forward(q, k, v)
    _r = fwd_check(o, ref, torch.float16)
    assert _r["ok"], _r


def test_small_head_dim_and_fp32_inputs(cuda_device):
    q, k, v = inputs(1, 2, 2, 700, 32, torch.float32, 33)
    o = _run(q, k, v, cuda_device)
    assert o.dtype == torch.float32 and o.shape == q.shape
    ref, _ = O.forward(q.bfloat16(), k.bfloat16(), v.bfloat16())
    _r = fwd_check(o.bfloat16(), ref, torch.bfloat16)
    assert _r["ok"], _r


def test_lse_and_relay_rows_through_c_abi(cuda_device):
    """Calls the C ABI directly: G rows / sources equal the oracle's top-k
    selection (exact), and the lse matches the oracle's."""
    from cron_root_attention import _lib
    L = _lib.lib()
    dev = cuda_device
    B, H, S, D = 1, 2, 3001, 128
    q, k, v = inputs(B, H, H, S, D, torch.bfloat16, 34)
    qd, kd, vd = (t.to(dev) for t in (q, k, v))
    W = L.cra_window(S)
    NB = (S + W - 1) // W
    NG = L.cra_global_rows(S, 1, 2)
    gk = torch.empty(B, H, NG, D, device=dev, dtype=torch.bfloat16)
    gv = torch.empty_like(gk)
    gsrc = torch.empty(B, H, NB, 2, device=dev, dtype=torch.int32)
    st = _lib.strides3
    s = torch.cuda.current_stream(dev).cuda_stream
    _lib.check(L.cra_relay_build(kd.data_ptr(), vd.data_ptr(), st(kd), st(vd), B, H, S, D, 1, 1, 2, None,
                                 gk.data_ptr(), gv.data_ptr(), gsrc.data_ptr(), s), "relay")
    o = torch.empty_like(qd)
    lse = torch.empty(B, H, S, device=dev, dtype=torch.float32)
    _lib.check(L.cra_fwd(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), gk.data_ptr(), gv.data_ptr(), st(qd), st(kd),
                         st(vd), B, H, H, S, D, 1, 1, 2, ctypes.c_float(D ** -0.5), o.data_ptr(), st(o),
                         lse.data_ptr(), None, s), "fwd")
    torch.cuda.synchronize(dev)
    ridx = O.relay_select(k, W, 2)
    assert torch.equal(gsrc.cpu().long(), ridx)
    rows = gk.cpu().view(B, H, NB, 3, D)
    idx = torch.arange(NB) * W
    assert torch.equal(rows[:, :, :, 0], k[:, :, idx])
    for t in range(2):
        assert torch.equal(rows[:, :, :, 1 + t], torch.gather(k, 2, ridx[..., t, None].expand(B, H, NB, D)))
    ref_o, ref_lse = O.forward(q, k, v)
    assert (lse.cpu() - ref_lse).abs().max().item() < 2e-3
    _r = fwd_check(o, ref_o, torch.bfloat16)
    assert _r["ok"], _r


def test_deterministic(cuda_device):
    q, k, v = inputs(1, 2, 2, 4100, 128, torch.bfloat16, 35)
    a = _run(q, k, v, cuda_device)
    b = _run(q, k, v, cuda_device)
    assert torch.equal(a, b)


def test_varlen_matches_per_document(cuda_device):
    cra = _cra()
    q, k, v = inputs(1, 2, 2, 5000, 64, torch.float16, 36)
    cu = [0, 1000, 3100, 5000]
    qd, kd, vd = (t.to(cuda_device) for t in (q, k, v))
    o = cra.cron_root_attention_varlen(qd, kd, vd, torch.tensor(cu))
    for s0, s1 in zip(cu, cu[1:]):
        ref, _ = O.forward(q[:, :, s0:s1], k[:, :, s0:s1], v[:, :, s0:s1])
        _r = fwd_check(o[:, :, s0:s1], ref, torch.float16)
        assert _r["ok"], _r


def test_varlen_equal_lengths_batched_matches_per_document(cuda_device):
    """Equal-length documents go through one batched call: forward equals the
    oracle, and forward and gradients equal separate per-document calls
    bit for bit (every (b, h) is computed independently)."""
    cra = _cra()
    q, k, v = inputs(1, 2, 2, 3700, 64, torch.float16, 37)
    cu = [0, 1024, 2048, 3072, 3700]
    qd, kd, vd = (t.to(cuda_device).requires_grad_(True) for t in (q, k, v))
    o = cra.cron_root_attention_varlen(qd, kd, vd, cu)
    g = torch.randn(o.shape, generator=torch.Generator().manual_seed(3)).to(o)
    (o * g).sum().backward()
    for s0, s1 in zip(cu, cu[1:]):
        ref, _ = O.forward(q[:, :, s0:s1], k[:, :, s0:s1], v[:, :, s0:s1])
        _r = fwd_check(o[:, :, s0:s1], ref, torch.float16)
        assert _r["ok"], _r
        qs, ks, vs = (t[:, :, s0:s1].detach().clone().requires_grad_(True) for t in (qd, kd, vd))
        os_ = cra.cron_root_attention(qs, ks, vs)
        (os_ * g[:, :, s0:s1]).sum().backward()
        assert torch.equal(os_, o[:, :, s0:s1])
        assert torch.equal(qs.grad, qd.grad[:, :, s0:s1])
        assert torch.equal(ks.grad, kd.grad[:, :, s0:s1])
        assert torch.equal(vs.grad, vd.grad[:, :, s0:s1])


def test_output_rows_only_16_byte_aligned(cuda_device):
    """Output rows 16- but not 32-byte aligned (row stride 136 elements): the
    kernels fall back from 32-byte to 16-byte stores; the result equals the
    one written into a contiguous output, bit for bit."""
    from cron_root_attention import _lib
    L = _lib.lib()
    dev = cuda_device
    B, H, S, D = 1, 2, 2600, 128
    q, k, v = (t.to(dev) for t in inputs(B, H, H, S, D, torch.bfloat16, 38))
    W = L.cra_window(S)
    NB = (S + W - 1) // W
    NG = L.cra_global_rows(S, 1, 2)
    gk = torch.empty(B, H, NG, D, device=dev, dtype=torch.bfloat16)
    gv = torch.empty_like(gk)
    gsrc = torch.empty(B, H, NB, 2, device=dev, dtype=torch.int32)
    st = _lib.strides3
    s = torch.cuda.current_stream(dev).cuda_stream
    _lib.check(L.cra_relay_build(k.data_ptr(), v.data_ptr(), st(k), st(v), B, H, S, D, 1, 1, 2, None,
                                 gk.data_ptr(), gv.data_ptr(), gsrc.data_ptr(), s), "relay")
    outs = []
    for wide in (D, 136):
        buf = torch.zeros(B, H, S, wide, device=dev, dtype=torch.bfloat16)
        o = buf[..., :D]
        lse = torch.empty(B, H, S, device=dev, dtype=torch.float32)
        _lib.check(L.cra_fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), gk.data_ptr(), gv.data_ptr(), st(q), st(k),
                             st(v), B, H, H, S, D, 1, 1, 2, ctypes.c_float(D ** -0.5), o.data_ptr(), st(o),
                             lse.data_ptr(), None, s), "fwd")
        outs.append((buf, o.clone()))
    torch.cuda.synchronize(dev)
    assert torch.equal(outs[0][1], outs[1][1])
    assert torch.count_nonzero(outs[1][0][..., D:]) == 0  # nothing written past the row


def test_varlen_mixed_lengths_one_launch_forward_backward(cuda_device):
    """Documents of different lengths (with and without the relay, one
    shorter than a tile, grouped K/V heads, a relay scale) through the
    single-launch varlen forward and the grouped backward, against the oracle
    per document."""
    cra = _cra()
    dev = cuda_device
    cu = [0, 100, 2600, 2700, 5300, 5429]  # lengths 100, 2500, 100, 2600, 129
    Hq, Hkv = 4, 2
    q, k, v, do = inputs(1, Hq, Hkv, cu[-1], 64, torch.bfloat16, 39, with_do=True)
    a = torch.tensor([0.2, -0.3])
    qd, kd, vd = (t.to(dev).requires_grad_(True) for t in (q, k, v))
    ad = a.to(dev).requires_grad_(True)
    o = cra.cron_root_attention_varlen(qd, kd, vd, cu, kv_groups=2, relay_log_scale=ad)
    o.backward(do.to(dev))
    torch.cuda.synchronize(dev)
    assert cra.check_device_errors(dev) == 0
    from parity import GRAD_REL_L2, rel_l2
    for s0, s1 in zip(cu, cu[1:]):
        sl = lambda t: t[:, :, s0:s1]
        ro, rdq, rdk, rdv, _ = O.forward_backward(sl(q), sl(k), sl(v), sl(do), kv_groups=2, relay_log_scale=a,
                                                  relay_dtype=torch.bfloat16)
        r = fwd_check(sl(o), ro, torch.bfloat16)
        assert r["ok"], (s0, r)
        for name, x, y in (("dq", sl(qd.grad), rdq), ("dk", sl(kd.grad), rdk), ("dv", sl(vd.grad), rdv)):
            assert rel_l2(x, y) <= GRAD_REL_L2, (s0, name, rel_l2(x, y))
    assert ad.grad is not None and torch.isfinite(ad.grad).all()
