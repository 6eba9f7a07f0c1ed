"""Tolerances of the GPU parity tests, stated once.

Forward (north_star: fp16/bf16 output vs the fp32 oracle, max-abs <= 2e-3 and
mean-abs <= 2e-4):
  * fp16 outputs are held to exactly that bar against the fp32 oracle.
  * bf16 outputs cannot meet it by construction.  Two roundings that the
    reference's own GPU path also performs dominate the error: the output
    itself (|o| reaches ~3 on rows near the sequence start, where one bf16 ulp
    is 1.6e-2), and P rounded to the value dtype before P.V (reference
    core.py:1027), whose error scales with |v| rather than |o|.  For bf16 the
    bar is applied beyond one bf16 ulp of those scales:
      |o - ref| <= 2e-3 + 2^-7 (|ref| + rms(v))   element-wise, and
      mean |o - ref| <= 2e-4 + mean |bf16(ref) - ref|
    (the second term is the mean error of the exact answer rounded to bf16).
Gradients (north_star): relative L2 error <= 1e-2 per tensor, against the
fp64 autograd restatement of the oracle.
"""
import os

import torch

FWD_MAX_ABS = 2e-3
FWD_MEAN_ABS = 2e-4
GRAD_REL_L2 = 1e-2


# Raw errors of every forward check of the session, printed by conftest.py
# in the terminal summary next to north_star's literal bar (2e-3 / 2e-4).
RECORDS = []


def fwd_check(o: torch.Tensor, ref: torch.Tensor, dtype: torch.dtype, v_rms: float = 1.0) -> dict:
    o = o.detach().float().cpu()
    ref = ref.float().cpu()
    err = (o - ref).abs()
    if dtype == torch.bfloat16:
        slack = (ref.abs() + v_rms) * 2.0 ** -7
        ok_max = bool((err <= FWD_MAX_ABS + slack).all())
        floor = (ref.to(torch.bfloat16).float() - ref).abs().mean().item()  # rounding the exact answer
        ok_mean = err.mean().item() <= FWD_MEAN_ABS + floor
    else:
        ok_max = err.max().item() <= FWD_MAX_ABS
        ok_mean = err.mean().item() <= FWD_MEAN_ABS
    r = {"ok": ok_max and ok_mean and not torch.isnan(o).any().item(),
         "max_abs": err.max().item(), "mean_abs": err.mean().item()}
    test = os.environ.get("PYTEST_CURRENT_TEST", "?").split(" ")[0]
    RECORDS.append((test, str(dtype).replace("torch.", ""), r["max_abs"], r["mean_abs"], r["ok"]))
    return r


def rel_l2(a: torch.Tensor, b: torch.Tensor) -> float:
    """||a - b|| / ||b||, with ||b|| floored at an RMS of 1e-3 so that an
    all-zero reference (e.g. dq at S = 1, where o = v_0) is judged by the
    absolute size of the error instead of dividing by zero."""
    a = a.detach().double().cpu()
    b = b.detach().double().cpu()
    floor = 1e-3 * b.numel() ** 0.5
    return ((a - b).norm() / max(b.norm().item(), floor)).item()


def inputs(B, Hq, Hkv, S, D, dtype, seed, sigma=1.0, with_do=False):
    """Seeded CPU inputs, drawn in fp32 in the order q, k, v, (dO), then cast."""
    g = torch.Generator().manual_seed(seed)
    q = (torch.randn(B, Hq, S, D, generator=g) * sigma).to(dtype)
    k = (torch.randn(B, Hkv, S, D, generator=g) * sigma).to(dtype)
    v = (torch.randn(B, Hkv, S, D, generator=g) * sigma).to(dtype)
    if with_do:
        do = torch.randn(B, Hq, S, D, generator=g).to(dtype)
        return q, k, v, do
    return q, k, v
