"""transformers integration (cron_root_attention.hf): registry entry, layout,
grouped K/V, scaling and the unsupported cases on CPU with the op replaced by
a recorder; on the GPU a small random-init Llama runs forward + backward
through the registry, and one layer's attention output is checked against
the oracle (replaces the reference's monkey-patch example,
examples/replace_huggingface.py:13-63)."""
import pytest
import torch

transformers = pytest.importorskip("transformers")

from cron_root_attention import core, hf  # noqa: E402


def _llama(layers=2, heads=2, kv_heads=1, head_dim=128, hidden=256, vocab=128, max_pos=4096):
    from transformers import LlamaConfig, LlamaForCausalLM

    cfg = LlamaConfig(vocab_size=vocab, hidden_size=hidden, intermediate_size=2 * hidden,
                      num_hidden_layers=layers, num_attention_heads=heads,
                      num_key_value_heads=kv_heads, head_dim=head_dim, max_position_embeddings=max_pos)
    return LlamaForCausalLM(cfg)


@pytest.fixture
def recorder(monkeypatch):
    calls = []

    def fake(q, k, v, kv_groups=1, **kw):
        calls.append({"q": q, "k": k, "v": v, "kv_groups": kv_groups})
        return q * 2.0

    monkeypatch.setattr(core, "cron_root_attention_v14", fake)
    return calls


def test_register_puts_the_function_in_the_registry():
    from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS

    assert hf.register() == "cron_root"
    assert ALL_ATTENTION_FUNCTIONS["cron_root"] is hf.cron_root_attention_forward
    assert hf.register("cra_alias") == "cra_alias"
    assert ALL_ATTENTION_FUNCTIONS["cra_alias"] is hf.cron_root_attention_forward


def test_layout_and_grouped_heads(recorder):
    m = torch.nn.Module()
    q = torch.randn(2, 4, 16, 64)
    k = torch.randn(2, 2, 16, 64)
    v = torch.randn(2, 2, 16, 64)
    out, w = hf.cron_root_attention_forward(m, q, k, v, None, scaling=64 ** -0.5)
    assert w is None
    assert out.shape == (2, 16, 4, 64) and out.is_contiguous()
    assert torch.equal(out, (q * 2.0).transpose(1, 2))
    (c,) = recorder
    assert c["kv_groups"] == 2 and c["k"] is k and c["v"] is v  # no K/V expansion


def test_other_scaling_is_folded_into_q(recorder):
    m = torch.nn.Module()
    q = torch.randn(1, 2, 8, 64)
    k = torch.randn(1, 2, 8, 64)
    hf.cron_root_attention_forward(m, q, k, k, None, scaling=0.25)
    assert torch.allclose(recorder[0]["q"], q * (0.25 / 64 ** -0.5))


@pytest.mark.parametrize("case", ["decode", "dropout", "noncausal", "heads"])
def test_unsupported_cases_raise(recorder, case):
    m = torch.nn.Module()
    q = torch.randn(1, 4, 8, 64)
    k = torch.randn(1, 2, 8, 64)
    if case == "decode":
        with pytest.raises(NotImplementedError):
            hf.cron_root_attention_forward(m, q[:, :, :1], k, k, None)
    elif case == "dropout":
        m.train()
        with pytest.raises(NotImplementedError):
            hf.cron_root_attention_forward(m, q, k, k, None, dropout=0.1)
        m.eval()
        hf.cron_root_attention_forward(m, q, k, k, None, dropout=0.1)  # inactive in eval
    elif case == "noncausal":
        with pytest.raises(NotImplementedError):
            hf.cron_root_attention_forward(m, q, k, k, None, is_causal=False)
    else:
        with pytest.raises(ValueError):
            hf.cron_root_attention_forward(m, q, torch.randn(1, 3, 8, 64), torch.randn(1, 3, 8, 64), None)
    assert len(recorder) == (1 if case == "dropout" else 0)


def test_llama_routes_every_layer_through_the_registry(recorder):
    hf.register()
    model = _llama(layers=3)
    model.set_attn_implementation("cron_root")
    ids = torch.randint(0, 128, (1, 32))
    logits = model(ids).logits
    assert logits.shape == (1, 32, 128)
    assert len(recorder) == 3
    assert all(c["kv_groups"] == 2 and c["k"].shape[1] == 1 for c in recorder)


@pytest.mark.gpu
def test_llama_forward_backward_on_gpu_matches_oracle(cuda_device):
    from oracle import cra_oracle as O
    from parity import fwd_check

    hf.register()
    seen = []

    def probe(module, query, key, value, attention_mask, **kw):
        out, w = hf.cron_root_attention_forward(module, query, key, value, attention_mask, **kw)
        if not seen:
            seen.append((query.detach(), key.detach(), value.detach(), out.detach()))
        return out, w

    from transformers import AttentionInterface

    AttentionInterface.register("cron_root_probe", probe)
    torch.manual_seed(0)
    model = _llama().to(device=cuda_device, dtype=torch.bfloat16)
    model.set_attn_implementation("cron_root_probe")
    S = 2304  # relay active (S > 2048)
    ids = torch.randint(0, 128, (1, S), device=cuda_device)
    out = model(ids, labels=ids)
    assert torch.isfinite(out.loss)
    out.loss.backward()
    grads = [p.grad for p in model.parameters() if p.grad is not None]
    assert grads and all(torch.isfinite(g).all() for g in grads)
    q, k, v, o = seen[0]
    ref, _ = O.forward(q.float().cpu(), k.float().cpu(), v.float().cpu(), kv_groups=q.shape[1] // k.shape[1],
                       relay_dtype=torch.bfloat16)
    res = fwd_check(o.transpose(1, 2), ref, torch.bfloat16, v_rms=v.float().pow(2).mean().sqrt().item())
    assert res["ok"], res


def test_causal_only_masks_are_accepted(recorder):
    m = torch.nn.Module()
    q = torch.randn(2, 2, 8, 64)
    tril = torch.ones(8, 8, dtype=torch.bool).tril()
    additive = torch.zeros(2, 1, 8, 8).masked_fill(~tril, torch.finfo(torch.float32).min)
    for mask in (None, tril.expand(2, 1, 8, 8), additive, torch.ones(2, 8, dtype=torch.long)):
        hf.cron_root_attention_forward(m, q, q, q, mask)
    assert len(recorder) == 4


def test_padding_masks_raise(recorder):
    m = torch.nn.Module()
    q = torch.randn(2, 2, 8, 64)
    pad = torch.ones(2, 8, dtype=torch.long)
    pad[1, :3] = 0  # left padding of the second sequence
    tril = torch.ones(8, 8, dtype=torch.bool).tril()
    keep4d = tril.expand(2, 1, 8, 8).clone()
    keep4d[1, :, :, :3] = False
    additive = torch.zeros(2, 1, 8, 8).masked_fill(~keep4d, torch.finfo(torch.float32).min)
    for mask in (pad, keep4d, additive):
        with pytest.raises(NotImplementedError, match="mask"):
            hf.cron_root_attention_forward(m, q, q, q, mask)
    assert recorder == []
