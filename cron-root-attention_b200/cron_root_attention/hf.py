"""Hugging Face transformers integration through the attention-interface registry.

The reference shows adoption by monkey-patching ``LlamaAttention.forward``
(examples/replace_huggingface.py:13-63): it re-implements the projections,
expands K/V for grouped-query attention with ``repeat_interleave`` and calls
``cron_root_attention``.  transformers >= 4.48 has a registry for exactly
this: ``AttentionInterface.register(name, fn)`` and then
``from_pretrained(..., attn_implementation=name)`` (or
``model.set_attn_implementation(name)``) routes every attention layer of any
model family through ``fn``.  This module provides that ``fn``:

    from cron_root_attention.hf import register
    register()                       # name "cron_root"
    model = AutoModelForCausalLM.from_config(cfg, attn_implementation="cron_root")

Semantics are the reference patch's: the attention is causal by
construction.  The model's mask is checked, not applied: a mask that only
restates causality (or none, which transformers passes when the batch has no
padding) is accepted; a mask that hides any key a causal query would see --
padding in a batch, packed documents -- raises ``NotImplementedError``, since
the kernels cannot honour it and silently ignoring it would give wrong
outputs.  Grouped K/V heads go to the kernels natively
(``kv_groups = H_q / H_kv``) instead of being expanded.  A model scaling other
than 1/sqrt(head_dim) is folded into q.  Unsupported, raising
``NotImplementedError``: attention dropout while training, a KV cache whose
key length differs from the query length (incremental decoding), and a call
that asks for non-causal attention.
"""
from __future__ import annotations

import math
from typing import Optional

import torch

from . import core as _core

ATTN_NAME = "cron_root"


def _hides_causal_keys(mask: torch.Tensor, S: int) -> bool:
    """True when ``mask`` masks out some (query i, key j <= i) pair.  Accepts
    a [B, S] keep-mask (1 = token present), or a [B, 1|H, S, S_k] boolean
    (True = attend) or additive float (0 = attend, large negative = masked)
    mask whose last S key columns align with the queries."""
    if mask.dim() == 2:  # padding mask
        return bool((mask[:, -S:] == 0).any())
    m = mask[..., -S:, -S:]
    tril = torch.ones(S, S, dtype=torch.bool, device=m.device).tril()
    if m.dtype == torch.bool:
        return bool((~m & tril).any())
    return bool(((m < -1e4) & tril).any())


def cron_root_attention_forward(module: torch.nn.Module, query: torch.Tensor, key: torch.Tensor,
                                value: torch.Tensor, attention_mask: Optional[torch.Tensor],
                                dropout: float = 0.0, scaling: Optional[float] = None,
                                is_causal: Optional[bool] = None, **kwargs):
    """Attention function with the signature transformers' registry expects.

    query: [B, H_q, S, D]; key, value: [B, H_kv, S, D].  Returns
    ``(out, None)`` with ``out`` [B, S, H_q, D] (the layout the model's output
    projection reshapes), and no attention weights.
    """
    if dropout and module.training:
        raise NotImplementedError("cron_root attention has no attention dropout")
    if is_causal is False:
        raise NotImplementedError("cron_root attention is causal only")
    if query.dim() != 4 or key.dim() != 4 or value.dim() != 4:
        raise ValueError("expected [B, H, S, D] query / key / value")
    B, Hq, S, D = query.shape
    if attention_mask is not None and _hides_causal_keys(attention_mask, S):
        raise NotImplementedError(
            "cron_root attention is causal only: the attention mask hides keys a causal query would see "
            "(padding or packed documents); use unpadded batches, or cron_root_attention_varlen for packing")
    Hkv = key.shape[1]
    if key.shape[2] != S or value.shape[2] != S:
        raise NotImplementedError(
            "cron_root attention needs the full sequence (query and key lengths "
            f"{S} vs {key.shape[2]}): incremental decoding with a KV cache is not supported")
    if Hq % Hkv != 0:
        raise ValueError(f"query heads {Hq} are not a multiple of key/value heads {Hkv}")
    if scaling is not None and not math.isclose(scaling, D ** -0.5, rel_tol=1e-6):
        query = query * (scaling / D ** -0.5)  # the kernels scale by 1/sqrt(D)
    out = _core.cron_root_attention_v14(query, key, value, kv_groups=Hq // Hkv)
    return out.transpose(1, 2).contiguous(), None


def register(name: str = ATTN_NAME) -> str:
    """Register :func:`cron_root_attention_forward` under ``name`` in
    transformers' ``AttentionInterface`` and return the name."""
    from transformers import AttentionInterface

    AttentionInterface.register(name, cron_root_attention_forward)
    return name
