"""Failure handling on the GPU without a fault: a bounded device wait that
runs out.  The test-only libcra_waitprobe.so (built with a 0.2 ms wait
limit) waits on an mbarrier nothing arrives at, using the same bounded-wait
code as every libcra kernel.  The wait must give up, record
CRA_DEV_WAIT_TIMEOUT (1) in the error word that check_device_errors reads,
raise the CTA's abort flag and exit; the context must stay usable, which a
normal forward checked against the oracle then shows."""
import ctypes
import os

import pytest
import torch

from oracle import cra_oracle as O
from parity import fwd_check, inputs

pytestmark = pytest.mark.gpu

PROBE = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "cron-root-attention_b200",
                     "cron_root_attention", "libcra_waitprobe.so")


def test_bounded_wait_times_out_and_context_survives(cuda_device):
    import cron_root_attention as cra
    from cron_root_attention.core import _err_word
    dev = cuda_device
    probe = ctypes.CDLL(PROBE)
    probe.cra_test_wait_timeout.restype = ctypes.c_int
    probe.cra_test_wait_timeout.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]
    assert cra.check_device_errors(dev) == 0
    out = torch.zeros(4, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    assert probe.cra_test_wait_timeout(_err_word(dev).data_ptr(), out.data_ptr(), 4, stream) == 0
    torch.cuda.synchronize(dev)
    assert out.tolist() == [3, 3, 3, 3]  # every CTA gave up with its abort flag set
    assert cra.check_device_errors(dev) == 1  # CRA_DEV_WAIT_TIMEOUT, and the word is cleared
    assert cra.check_device_errors(dev) == 0
    # the context is still usable: a normal call of the real library is correct
    q, k, v = inputs(1, 1, 1, 300, 64, torch.float16, 70)
    o = cra.cron_root_attention(q.to(dev), k.to(dev), v.to(dev))
    torch.cuda.synchronize(dev)
    assert cra.check_device_errors(dev) == 0
    ref, _ = O.forward(q, k, v)
    r = fwd_check(o, ref, torch.float16)
    assert r["ok"], r
