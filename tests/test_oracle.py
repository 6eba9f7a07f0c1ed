"""CPU tests of the oracle: pinned to the reference's own outputs (golden
fixtures made by tests/golden/make_golden.py from cra_cpu_fast), cross-checked
against an independent dense-mask statement, and the backward restatement
pinned through its forward."""
import glob
import os

import numpy as np
import pytest
import torch

from oracle import cra_oracle as O

GOLDEN = sorted(glob.glob(os.path.join(os.path.dirname(__file__), "golden", "*.npz")))


def load_golden(path):
    z = np.load(path)
    dt = str(z["dtype"])

    def t(a):
        if dt == "bf16":
            return torch.from_numpy(a.view(np.int16)).view(torch.bfloat16)
        return torch.from_numpy(a)

    B, H, S, D, use_relay, seed = (int(x) for x in z["meta"])
    return t(z["q"]), t(z["k"]), t(z["v"]), torch.from_numpy(z["out"]), bool(use_relay)


def test_golden_fixtures_present():
    assert len(GOLDEN) >= 4


@pytest.mark.parametrize("path", GOLDEN, ids=[os.path.basename(p) for p in GOLDEN])
def test_oracle_matches_reference_golden(path):
    q, k, v, out, use_relay = load_golden(path)
    o32, _ = O.forward(q, k, v, use_relay=use_relay, dtype=torch.float32)
    assert (o32 - out).abs().max().item() <= 1e-5
    o64, _ = O.forward(q, k, v, use_relay=use_relay, dtype=torch.float64)
    assert (o64 - out.double()).abs().max().item() <= 1e-4


@pytest.mark.parametrize("S", [1, 2, 3, 16, 17, 255, 256, 257, 2048, 2049, 2500, 4097])
def test_oracle_vs_dense_statement(S):
    g = torch.Generator().manual_seed(S)
    q, k, v = (torch.randn(1, 2, S, 16, generator=g, dtype=torch.float64) for _ in range(3))
    o, _ = O.forward(q, k, v, dtype=torch.float64)
    d = O.dense_forward(q, k, v)
    assert (o - d).abs().max().item() < 1e-12


@pytest.mark.parametrize("top_k", [1, 3, 4])
def test_oracle_topk_variants_vs_dense(top_k):
    g = torch.Generator().manual_seed(top_k)
    q, k, v = (torch.randn(1, 1, 2300, 16, generator=g, dtype=torch.float64) for _ in range(3))
    o, _ = O.forward(q, k, v, top_k=top_k, dtype=torch.float64)
    d = O.dense_forward(q, k, v, top_k=top_k)
    assert (o - d).abs().max().item() < 1e-12


def test_lse_consistent():
    g = torch.Generator().manual_seed(5)
    q, k, v = (torch.randn(1, 1, 2600, 16, generator=g, dtype=torch.float64) for _ in range(3))
    o, lse = O.forward(q, k, v, dtype=torch.float64)
    # row 0 sees only itself: lse = q.k * scale
    assert abs(lse[0, 0, 0].item() - (q[0, 0, 0] @ k[0, 0, 0]).item() / 4.0) < 1e-12


@pytest.mark.parametrize("S,kv_groups,alpha", [(300, 1, False), (2400, 1, False), (2400, 2, True), (2100, 1, True)])
def test_backward_restatement_forward_equals_oracle(S, kv_groups, alpha):
    g = torch.Generator().manual_seed(S)
    Hq = 2 * kv_groups
    q = torch.randn(1, Hq, S, 16, generator=g, dtype=torch.float64)
    k, v = (torch.randn(1, 2, S, 16, generator=g, dtype=torch.float64) for _ in range(2))
    do = torch.randn(1, Hq, S, 16, generator=g, dtype=torch.float64)
    a = torch.randn(2, generator=g, dtype=torch.float64) * 0.3 if alpha else None
    o1, _ = O.forward(q, k, v, kv_groups=kv_groups, relay_log_scale=a, dtype=torch.float64)
    o2, dq, dk, dv, da = O.forward_backward(q, k, v, do, kv_groups=kv_groups, relay_log_scale=a)
    assert (o1 - o2).abs().max().item() < 1e-12
    assert dq.shape == q.shape and dk.shape == k.shape and dv.shape == v.shape
    # size-independent identities used by the full-size GPU tests (they hold
    # without a relay scale: softmax rows sum to 1, and sum_j dS_qj = 0)
    if a is None:
        assert (dv.sum(2) - do.view(1, 2, kv_groups, S, 16).sum((2, 3))).abs().max().item() < 1e-9
        assert dk.sum(2).abs().max().item() < 1e-9


def test_backward_restatement_gradcheck():
    """Autograd of the restatement's math equals finite differences."""
    g = torch.Generator().manual_seed(0)
    q, k, v = (torch.randn(1, 1, 12, 4, generator=g, dtype=torch.float64, requires_grad=True) for _ in range(3))

    def f(q, k, v):
        B, H, S, D = q.shape
        W = O.window(S)
        gl = O.build_global_list(k.detach(), W, True, 2)
        Kg = O._gather_rows(k, gl.idx)
        Vg = O._gather_rows(v, gl.idx)
        pos = torch.arange(S)
        qp, kp = pos.view(-1, 1), pos.view(1, -1)
        ls = (qp - W + 1).clamp(min=0)
        m_l = (kp <= qp) & (kp >= qp - W + 1)
        m_g = gl.visible_before.view(1, -1) < ls
        s_l = (q @ k.transpose(-1, -2) / 2.0).masked_fill(~m_l, float("-inf"))
        s_g = (q @ Kg.transpose(-1, -2) / 2.0).masked_fill(~m_g, float("-inf"))
        p = torch.softmax(torch.cat([s_l, s_g], -1), -1)
        return p[..., :S] @ v + p[..., S:] @ Vg

    assert torch.autograd.gradcheck(f, (q, k, v))


def test_relay_select_ties_lowest_index():
    k = torch.zeros(1, 1, 9, 2, dtype=torch.float64)  # W = 3
    k[0, 0, 1] = torch.tensor([1.0, 0.0])
    k[0, 0, 2] = torch.tensor([0.0, 1.0])  # equal norm to row 1 -> row 1 first
    k[0, 0, 4] = torch.tensor([2.0, 0.0])
    idx = O.relay_select(k, 3, 2)
    assert idx[0, 0, 0].tolist() == [1, 2]
    assert idx[0, 0, 1].tolist() == [4, 3]  # zero rows 3 and 5 tie -> 3
    assert idx[0, 0, 2].tolist() == [6, 7]


def test_visible_pair_counts_match_flop_accounting():
    assert O.visible_pairs(4096) == 639262
    assert O.visible_pairs(16384) == 5177918
    assert O.visible_pairs(65536) == 41682046
    assert O.window(524288) == 725
    assert O.visible_pairs(524288) == 946727290


def test_window_and_threshold():
    assert [O.window(s) for s in (1, 2, 4, 5, 16, 17, 65536, 65537)] == [1, 2, 2, 3, 4, 5, 256, 257]
    assert not O.relay_active(2048) and O.relay_active(2049)
