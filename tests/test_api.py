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


def test_varlen_groups_equal_lengths_into_one_call(monkeypatch):
    """Equal-length documents run as one batched call; the result equals the
    per-document computation (op replaced by the CPU oracle here)."""
    import torch
    import cron_root_attention as cra
    from cron_root_attention import core
    from oracle import cra_oracle as O

    calls = []

    def oracle_op(q, k, v, use_persistent=False, kv_groups=1, relay_log_scale=None, relay_top_k=2):
        calls.append(tuple(q.shape))
        return O.forward(q, k, v, kv_groups=kv_groups, top_k=relay_top_k, dtype=torch.float64)[0]

    monkeypatch.setattr(core, "cron_root_attention_v14", oracle_op)
    g = torch.Generator().manual_seed(5)
    lens = [300, 120, 300, 0, 57, 120, 300]
    S = sum(lens)
    cu = [0]
    for n in lens:
        cu.append(cu[-1] + n)
    q = torch.randn(2, 4, S, 16, generator=g, dtype=torch.float64)
    k = torch.randn(2, 2, S, 16, generator=g, dtype=torch.float64)
    v = torch.randn(2, 2, S, 16, generator=g, dtype=torch.float64)
    o = cra.cron_root_attention_varlen(q, k, v, cu, kv_groups=2)
    assert sorted(calls) == sorted([(6, 4, 300, 16), (4, 4, 120, 16), (2, 4, 57, 16)])
    for s0, s1 in zip(cu, cu[1:]):
        if s1 > s0:
            ref = O.forward(q[:, :, s0:s1], k[:, :, s0:s1], v[:, :, s0:s1], kv_groups=2, dtype=torch.float64)[0]
            assert (o[:, :, s0:s1] - ref).abs().max().item() < 1e-12
