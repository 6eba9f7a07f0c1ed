"""Length-based backend selection (reference cron_root_attention/hybrid.py).

``backend="sdpa"`` and ``"auto"`` below ``threshold`` keep the reference's
documented meaning (torch's causal scaled_dot_product_attention); the sqrt(N)
op itself never dispatches anywhere else.
"""
from typing import Literal

import torch
import torch.nn as nn
import torch.nn.functional as F

from .core import cron_root_attention_v14

_SDPA_THRESHOLD = 1536  # reference hybrid.py:22


def cron_root_attention_hybrid(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                               backend: Literal["auto", "cron_root", "sdpa"] = "auto",
                               threshold: int = _SDPA_THRESHOLD) -> torch.Tensor:
    """Reference hybrid.py:25-64: "cron_root" forces the sqrt(N) op, "sdpa"
    forces dense causal SDPA, "auto" picks the sqrt(N) op when S >= threshold."""
    S = q.shape[2]
    if backend == "cron_root":
        return cron_root_attention_v14(q, k, v)
    if backend == "sdpa":
        return F.scaled_dot_product_attention(q, k, v, is_causal=True)
    if S >= threshold:
        return cron_root_attention_v14(q, k, v)
    return F.scaled_dot_product_attention(q, k, v, is_causal=True)


class CronRootAttentionHybrid(nn.Module):
    """Reference hybrid.py:67-124."""

    def __init__(self, d_model: int, n_heads: int, threshold: int = _SDPA_THRESHOLD,
                 dropout: float = 0.0, bias: bool = False):
        super().__init__()
        self.d_model = d_model
        self.n_heads = n_heads
        self.head_dim = d_model // n_heads
        self.threshold = threshold
        self.dropout = dropout
        self.q_proj = nn.Linear(d_model, d_model, bias=bias)
        self.k_proj = nn.Linear(d_model, d_model, bias=bias)
        self.v_proj = nn.Linear(d_model, d_model, bias=bias)
        self.o_proj = nn.Linear(d_model, d_model, bias=bias)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        B, S, D = x.shape
        q = self.q_proj(x).view(B, S, self.n_heads, self.head_dim).transpose(1, 2)
        k = self.k_proj(x).view(B, S, self.n_heads, self.head_dim).transpose(1, 2)
        v = self.v_proj(x).view(B, S, self.n_heads, self.head_dim).transpose(1, 2)
        out = cron_root_attention_hybrid(q, k, v, backend="auto", threshold=self.threshold)
        out = self.o_proj(out.transpose(1, 2).contiguous().view(B, S, D))
        if self.dropout > 0 and self.training:
            out = F.dropout(out, p=self.dropout)
        return out
