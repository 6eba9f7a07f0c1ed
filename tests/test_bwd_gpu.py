"""Backward parity of the CUDA path against the fp64 autograd restatement of
the oracle (relative L2 <= 1e-2 per gradient), plus size-independent
identities at the BASELINE training size."""
import pytest
import torch

from oracle import cra_oracle as O
from parity import GRAD_REL_L2, fwd_check, inputs, rel_l2

pytestmark = pytest.mark.gpu


def _grads(q, k, v, do, dev, **kw):
    import cron_root_attention as cra
    qd, kd, vd = (t.to(dev).requires_grad_(True) for t in (q, k, v))
    a = kw.pop("relay_log_scale", None)
    ad = a.to(dev).requires_grad_(True) if a is not None else None
    o = cra.cron_root_attention(qd, kd, vd, relay_log_scale=ad, **kw)
    o.backward(do.to(dev))
    torch.cuda.synchronize(dev)
    assert cra.check_device_errors(dev) == 0
    return o.detach(), qd.grad, kd.grad, vd.grad, (ad.grad if ad is not None else None)


CASES = [
    # B, Hq, Hkv, S, D, dtype, seed, top_k, alpha
    (1, 2, 2, 1, 64, torch.float16, 0, 2, False),
    (1, 1, 1, 17, 64, torch.bfloat16, 1, 2, False),
    (1, 2, 2, 300, 64, torch.float16, 2, 2, False),
    (1, 2, 2, 2304, 64, torch.float16, 3, 2, False),
    (1, 1, 1, 3001, 128, torch.bfloat16, 4, 2, False),
    (1, 4, 2, 2500, 64, torch.bfloat16, 5, 2, False),
    (1, 2, 2, 2600, 128, torch.float16, 6, 2, True),
    (2, 2, 2, 4100, 128, torch.bfloat16, 7, 2, False),
    (1, 2, 2, 2200, 128, torch.float16, 8, 1, False),
    (1, 2, 2, 2200, 64, torch.float16, 9, 3, False),
]


@pytest.mark.parametrize("B,Hq,Hkv,S,D,dt,seed,top_k,alpha", CASES)
def test_backward_vs_restatement(B, Hq, Hkv, S, D, dt, seed, top_k, alpha, cuda_device):
    q, k, v, do = inputs(B, Hq, Hkv, S, D, dt, seed, with_do=True)
    a = torch.linspace(-0.4, 0.4, Hkv) if alpha else None
    o, dq, dk, dv, da = _grads(q, k, v, do, cuda_device, kv_groups=Hq // Hkv, relay_top_k=top_k,
                               relay_log_scale=a)
    ro, rdq, rdk, rdv, rda = O.forward_backward(q, k, v, do, kv_groups=Hq // Hkv, top_k=top_k,
                                                relay_log_scale=a, relay_dtype=dt if alpha else None)
    _r = fwd_check(o, ro, dt)
    assert _r["ok"], _r
    for name, x, y in (("dq", dq, rdq), ("dk", dk, rdk), ("dv", dv, rdv)):
        assert rel_l2(x, y) <= GRAD_REL_L2, (name, rel_l2(x, y))
    if alpha:
        assert rel_l2(da, rda) <= GRAD_REL_L2


def test_backward_deterministic(cuda_device):
    q, k, v, do = inputs(1, 2, 2, 4100, 128, torch.bfloat16, 11, with_do=True)
    r1 = _grads(q, k, v, do, cuda_device)
    r2 = _grads(q, k, v, do, cuda_device)
    for a, b in zip(r1[:4], r2[:4]):
        assert torch.equal(a, b)


def test_stride_zero_grad_output(cuda_device):
    """o.sum().backward() hands the op an expanded (stride-0) dO."""
    import cron_root_attention as cra
    q, k, v = inputs(1, 2, 2, 2500, 64, torch.float16, 12)
    qd, kd, vd = (t.to(cuda_device).requires_grad_(True) for t in (q, k, v))
    cra.cron_root_attention(qd, kd, vd).float().sum().backward()
    ones = torch.ones(1, 2, 2500, 64, dtype=torch.float16)
    _, rdq, rdk, rdv, _ = O.forward_backward(q, k, v, ones)
    for x, y in ((qd.grad, rdq), (kd.grad, rdk), (vd.grad, rdv)):
        assert rel_l2(x, y) <= GRAD_REL_L2


def test_config3_full_size(cuda_device):
    """B2 H16 D128 S65536 bf16, seed 2, dO ~ N(0,1).
    (a) Eight whole (b, h) slices -- every row -- of o, dq, dk, dv against the
    fp32 oracle restatement (the backward restatement is exact for dk / dv
    only with every query row, hence whole slices); (b) identities that hold
    at any size over all (b, h): sum_j dV_j = sum_q dO_q, sum_j dK_j = 0."""
    dev = cuda_device
    B, H, S, D = 2, 16, 65536, 128
    q, k, v, do = inputs(B, H, H, S, D, torch.bfloat16, 2, with_do=True)
    o, dq, dk, dv, _ = _grads(q, k, v, do, dev)
    assert not any(torch.isnan(t).any().item() for t in (o, dq, dk, dv))
    sdv = dv.double().sum(2).cpu()
    sdo = do.double().sum(2)
    assert rel_l2(sdv, sdo) <= GRAD_REL_L2
    # bf16 rounding of dK alone leaves ~2e-3 of this ratio
    assert (dk.double().sum(2).cpu().norm() / dk.double().norm().cpu()).item() <= 1e-2
    torch.set_num_threads(max(1, torch.get_num_threads()))
    for b, h in ((1, 5), (0, 15), (0, 0), (1, 1), (0, 7), (1, 10), (0, 12), (1, 14)):
        sl = lambda t: t[b:b + 1, h:h + 1]
        ro, rdq, rdk, rdv, _ = O.forward_backward(sl(q), sl(k), sl(v), sl(do), dtype=torch.float32)
        _r = fwd_check(sl(o), ro, torch.bfloat16)
        assert _r["ok"], _r
        for name, x, y in (("dq", sl(dq), rdq), ("dk", sl(dk), rdk), ("dv", sl(dv), rdv)):
            assert rel_l2(x, y) <= GRAD_REL_L2, (name, rel_l2(x, y))


@pytest.mark.parametrize("B,Hq,Hkv,S,dt,seed", [(2, 2, 2, 4100, torch.bfloat16, 7), (1, 4, 2, 2500, torch.float16, 5),
                                               (1, 2, 2, 300, torch.bfloat16, 3)])
def test_fused_backward_through_c_abi(B, Hq, Hkv, S, dt, seed, cuda_device):
    """cra_bwd_fused (dQ from the key passes by atomic adds) against the
    oracle, and dk / dv bit for bit equal to cra_bwd's."""
    import ctypes
    import cron_root_attention as cra
    from cron_root_attention import _lib
    L = _lib.lib()
    dev = cuda_device
    D = 128
    q, k, v, do = inputs(B, Hq, Hkv, S, D, dt, seed, with_do=True)
    qd, kd, vd, dod = (t.to(dev) for t in (q, k, v, do))
    qd.requires_grad_(True), kd.requires_grad_(True), vd.requires_grad_(True)
    o = cra.cron_root_attention(qd, kd, vd, kv_groups=Hq // Hkv)
    o.backward(dod, retain_graph=True)
    ctx = o.grad_fn
    qc, kc, vc, oc, lse, gk, gv, gsrc, _ = ctx.saved_tensors
    st = _lib.strides3
    use_relay = int(S > 2048)
    outs = [torch.empty_like(t) for t in (qc, kc, vc)]
    ws_b = L.cra_bwd_fused_workspace_bytes(B, Hq, Hkv, S, D, use_relay, 2)
    assert ws_b > L.cra_bwd_workspace_bytes(B, Hq, Hkv, S, D, use_relay, 2)
    ws = torch.empty(ws_b, device=dev, dtype=torch.uint8)
    s = torch.cuda.current_stream(dev).cuda_stream
    _lib.check(L.cra_bwd_fused(qc.data_ptr(), kc.data_ptr(), vc.data_ptr(), oc.data_ptr(), dod.data_ptr(),
                               lse.data_ptr(), gk.data_ptr(), gv.data_ptr(), gsrc.data_ptr(), st(qc), st(kc), st(vc),
                               st(oc), st(dod), B, Hq, Hkv, S, D, 1 if dt == torch.bfloat16 else 0, use_relay, 2,
                               ctypes.c_float(D ** -0.5), None, outs[0].data_ptr(), outs[1].data_ptr(),
                               outs[2].data_ptr(), st(outs[0]), st(outs[1]), st(outs[2]), None, ws.data_ptr(), ws_b,
                               None, s), "cra_bwd_fused")
    torch.cuda.synchronize(dev)
    assert cra.check_device_errors(dev) == 0
    _, rdq, rdk, rdv, _ = O.forward_backward(q, k, v, do, kv_groups=Hq // Hkv)
    for name, x, y in (("dq", outs[0], rdq), ("dk", outs[1], rdk), ("dv", outs[2], rdv)):
        assert rel_l2(x, y) <= GRAD_REL_L2, (name, rel_l2(x, y))
    assert torch.equal(outs[1], kd.grad) and torch.equal(outs[2], vd.grad)
    assert rel_l2(outs[0], qd.grad) <= 1e-3
