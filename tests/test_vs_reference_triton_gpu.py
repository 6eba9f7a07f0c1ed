"""This implementation against the reference's own GPU path (its Triton
kernels, the unmodified package installed in baseline/_ref, git-ignored) on
the same inputs: forward output and the three gradients.  Skipped when
baseline/_ref holds no install of the reference.

The reference runs in a child process (its package has this repository's
package name) and saves its results; both sides are bf16 / fp16 results of
the same fp32-accumulated math, so the bars are two 16-bit ulps of the
output's scale and a relative L2 for the gradients (the reference adds its strided
and relay key gradients with 16-bit atomics, core.py:1886-1888,
2095-2097)."""
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "baseline", "_ref")

_CHILD = r"""
import sys
import torch
ref, path = sys.argv[1], sys.argv[2]
sys.path.insert(0, ref)
import cron_root_attention as R
assert R.__file__.startswith(ref), R.__file__
d = torch.load(path)
dev = torch.device("cuda", 0)
q, k, v, do = (d[n].to(dev).requires_grad_(n != "do") for n in ("q", "k", "v", "do"))
o = R.cron_root_attention(q, k, v)
o.backward(do)
torch.save({"o": o.detach().cpu(), "dq": q.grad.cpu(), "dk": k.grad.cpu(), "dv": v.grad.cpu()}, path + ".out")
"""


@pytest.mark.skipif(not os.path.isdir(os.path.join(REF, "cron_root_attention")),
                    reason="no install of the reference in baseline/_ref")
@pytest.mark.parametrize("S,D,dt", [(4096, 128, torch.bfloat16), (3000, 64, torch.float16), (1500, 128, torch.bfloat16)])
def test_matches_reference_gpu_path(S, D, dt, cuda_device, tmp_path):
    g = torch.Generator().manual_seed(S + D)
    B, H = 1, 2
    q, k, v, do = (torch.randn(B, H, S, D, generator=g).to(dt) for _ in range(4))
    path = str(tmp_path / "inputs.pt")
    torch.save({"q": q, "k": k, "v": v, "do": do}, path)
    r = subprocess.run([sys.executable, "-c", _CHILD, REF, path], capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stderr[-2000:]
    ref = torch.load(path + ".out")

    from cron_root_attention import cron_root_attention
    qd, kd, vd = (t.to(cuda_device).requires_grad_(True) for t in (q, k, v))
    o = cron_root_attention(qd, kd, vd)
    o.backward(do.to(cuda_device))
    torch.cuda.synchronize()

    # two independently rounded 16-bit results of a convex combination of v
    # rows: within two ulps of the output's scale (|o| + rms v) of each other
    ulp = 2.0 ** -7 if dt == torch.bfloat16 else 2.0 ** -10
    a, b = o.detach().float().cpu(), ref["o"].float()
    rms_v = v.float().pow(2).mean().sqrt().item()
    err = (a - b).abs()
    assert (err <= 2e-3 + 2 * ulp * (b.abs() + rms_v)).all(), err.max().item()
    assert err.mean().item() <= 5e-4, err.mean().item()
    for n, t in (("dq", qd.grad), ("dk", kd.grad), ("dv", vd.grad)):
        x, y = t.float().cpu(), ref[n].float()
        rel = ((x - y).norm() / y.norm()).item()
        assert rel < 2e-2, (n, rel)
