"""The reference package's own smoke tests (reference tests/test_attention.py:
shapes, NaN/Inf, fp32 backward with head_dim 32, modules, hybrid backends,
GPU info, sub-quadratic scaling), re-run against this implementation."""
import time

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture
def dev(cuda_device):
    return cuda_device


def test_forward_shape_and_dtype(dev):
    from cron_root_attention import cron_root_attention
    q, k, v = (torch.randn(2, 4, 256, 64, device=dev, dtype=torch.float16) for _ in range(3))
    out = cron_root_attention(q, k, v)
    assert out.shape == (2, 4, 256, 64) and out.dtype == torch.float16


def test_no_nan_inf(dev):
    from cron_root_attention import cron_root_attention
    q, k, v = (torch.randn(1, 8, 512, 64, device=dev, dtype=torch.float16) for _ in range(3))
    out = cron_root_attention(q, k, v)
    assert torch.isfinite(out).all()


def test_fp32_backward_shapes_and_finite(dev):
    from cron_root_attention import cron_root_attention
    q, k, v = (torch.randn(1, 2, 256, 32, device=dev, requires_grad=True) for _ in range(3))
    out = cron_root_attention(q, k, v)
    out.backward(torch.randn_like(out))
    for t in (q, k, v):
        assert t.grad is not None and t.grad.shape == t.shape and torch.isfinite(t.grad).all()


def test_module_api(dev):
    from cron_root_attention import CronRootAttention
    attn = CronRootAttention(d_model=512, n_heads=8).to(dev).half()
    x = torch.randn(2, 256, 512, device=dev, dtype=torch.float16)
    assert attn(x).shape == x.shape
    gqa = CronRootAttention(d_model=512, n_heads=8, n_kv_heads=2).to(dev).half()
    y = gqa(x)
    y.float().sum().backward()
    assert gqa.k_proj.weight.grad is not None


def test_multihead_api(dev):
    from cron_root_attention import CronRootMultiheadAttention
    mha = CronRootMultiheadAttention(embed_dim=512, num_heads=8, batch_first=True).to(dev).half()
    x = torch.randn(2, 256, 512, device=dev, dtype=torch.float16)
    out, w = mha(x, x, x)
    assert out.shape == x.shape and w is None


def test_gpu_info(dev):
    from cron_root_attention import get_gpu_info, get_num_sms
    info = get_gpu_info()
    assert info["sm_count"] == get_num_sms() > 0


@pytest.mark.parametrize("backend", ["auto", "cron_root", "sdpa"])
def test_hybrid_backends(backend, dev):
    from cron_root_attention import cron_root_attention_hybrid
    q, k, v = (torch.randn(1, 4, 2048, 64, device=dev, dtype=torch.float16) for _ in range(3))
    assert cron_root_attention_hybrid(q, k, v, backend=backend).shape == q.shape


def test_subquadratic_scaling(dev):
    """T(16K) / T(4K) well below the 16x a dense kernel would need."""
    from cron_root_attention import cron_root_attention

    def t(S):
        q, k, v = (torch.randn(1, 8, S, 64, device=dev, dtype=torch.float16) for _ in range(3))
        for _ in range(3):
            cron_root_attention(q, k, v)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(10):
            cron_root_attention(q, k, v)
        torch.cuda.synchronize()
        return time.perf_counter() - t0

    assert t(16384) / t(4096) < 16
