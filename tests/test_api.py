"""CPU tests of the Python API surface (same public names as the reference
package's __init__.py:208-222) and of its no-CPU-fallback rule."""
import pytest
import torch


def test_public_names():
    import cron_root_attention as cra
    for n in ["cron_root_attention", "cron_root_attention_v14", "cron_root_attention_varlen",
              "warmup_varlen_shapes", "CronRootAttention", "CronRootMultiheadAttention",
              "cron_root_attention_hybrid", "CronRootAttentionHybrid", "calibrate", "get_num_sms",
              "get_gpu_info", "GPU_SM_MAP", "__version__"]:
        assert n in cra.__all__ and hasattr(cra, n)
    assert cra.cron_root_attention is cra.cron_root_attention_v14
    assert cra.GPU_SM_MAP["NVIDIA B200"] == 148


def test_cpu_tensors_raise_no_fallback():
    import cron_root_attention as cra
    q = torch.randn(1, 2, 64, 64)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        cra.cron_root_attention(q, q, q)


def test_modules_construct():
    import cron_root_attention as cra
    m = cra.CronRootAttention(d_model=256, n_heads=4, n_kv_heads=2)
    assert m.kv_groups == 2 and m.k_proj.out_features == 128
    mha = cra.CronRootMultiheadAttention(embed_dim=128, num_heads=2)
    assert mha.in_proj_weight.shape == (384, 128)


def test_hybrid_sdpa_branch_on_cpu():
    import cron_root_attention as cra
    q = torch.randn(1, 2, 64, 32)
    out = cra.cron_root_attention_hybrid(q, q, q, backend="auto")  # S < threshold -> SDPA
    ref = torch.nn.functional.scaled_dot_product_attention(q, q, q, is_causal=True)
    assert torch.allclose(out, ref)


def test_varlen_rejects_device_cu_seqlens_and_bad_bounds():
    import cron_root_attention as cra
    q = torch.randn(1, 1, 10, 64)
    with pytest.raises(ValueError):
        cra.cron_root_attention_varlen(q, q, q, [0, 4, 9])


def test_gpu_info_without_gpu():
    import cron_root_attention as cra
    if not torch.cuda.is_available():
        assert cra.get_gpu_info()["sm_count"] == 0
        assert cra.get_num_sms() == 1


def test_varlen_argument_checks():
    """cu_seqlens must start at 0, end at the packed length and not decrease,
    and live on the host; CPU tensors are refused (no CPU fallback)."""
    import pytest
    import torch
    import cron_root_attention as cra
    q = torch.zeros(1, 2, 10, 16)
    for bad in ([1, 10], [0, 9], [0, 6, 4, 10]):
        with pytest.raises(ValueError):
            cra.cron_root_attention_varlen(q, q, q, bad)
    with pytest.raises(RuntimeError, match="CUDA"):
        cra.cron_root_attention_varlen(q, q, q, [0, 4, 10])
