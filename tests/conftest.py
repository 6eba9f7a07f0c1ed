import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "cron-root-attention_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200) device")


@pytest.fixture(scope="session")
def cuda_device():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("CUDA not available")
    return torch.device("cuda", 0)


def pytest_terminal_summary(terminalreporter):
    """Raw forward errors against the fp32/fp64 oracle, beside north_star's
    literal bar (max-abs 2e-3, mean-abs 2e-4).  fp16 checks use that bar; bf16
    checks use the bar beyond one bf16 ulp stated in tests/parity.py, so their
    raw numbers can exceed the literal one."""
    try:
        import parity
    except ImportError:
        return
    if not parity.RECORDS:
        return
    tr = terminalreporter
    tr.section("forward parity: raw errors vs the oracle (north_star bar: max-abs 2e-3, mean-abs 2e-4)")
    worst = {}
    for test, dt, mx, mean, ok in parity.RECORDS:
        w = worst.get((test, dt))
        if w is None or mx > w[0]:
            worst[(test, dt)] = (mx, mean, ok)
    for (test, dt), (mx, mean, ok) in sorted(worst.items()):
        lit = "within" if (mx <= 2e-3 and mean <= 2e-4) else "beyond"
        tr.write_line(f"{dt:9s} max_abs {mx:.3e} mean_abs {mean:.3e} ({lit} the literal bar; "
                      f"{'pass' if ok else 'FAIL'} at the test's bar)  {test}")
