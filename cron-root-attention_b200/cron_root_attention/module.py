"""nn.Module wrappers (reference cron_root_attention/module.py).

``CronRootAttention`` (reference module.py:20-126) and
``CronRootMultiheadAttention`` (reference module.py:129-247): projections and
reshapes around ``cron_root_attention_v14``, same constructor arguments,
same forward signatures and return values.  Grouped K/V heads (GQA) are
passed to the op natively via ``kv_groups`` instead of being expanded.
"""
from typing import Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from .core import cron_root_attention_v14


class CronRootAttention(nn.Module):
    """sqrt(N) sparse self/cross attention layer with q/k/v/o projections.

    Args: d_model, n_heads, n_kv_heads (GQA, default n_heads), dropout, bias.
    forward(x, kv=None) -> [B, S, d_model]
    """

    def __init__(self, d_model: int, n_heads: int, n_kv_heads: Optional[int] = None,
                 dropout: float = 0.0, bias: bool = False):
        super().__init__()
        self.d_model = d_model
        self.n_heads = n_heads
        self.n_kv_heads = n_kv_heads or n_heads
        self.head_dim = d_model // n_heads
        self.dropout = dropout
        assert d_model % n_heads == 0, "d_model must be divisible by n_heads"
        assert n_heads % self.n_kv_heads == 0, "n_heads must be divisible by n_kv_heads"
        self.kv_groups = n_heads // self.n_kv_heads
        self.drop = nn.Dropout(dropout) if dropout > 0 else nn.Identity()
        self.q_proj = nn.Linear(d_model, d_model, bias=bias)
        self.k_proj = nn.Linear(d_model, self.n_kv_heads * self.head_dim, bias=bias)
        self.v_proj = nn.Linear(d_model, self.n_kv_heads * self.head_dim, bias=bias)
        self.o_proj = nn.Linear(d_model, d_model, bias=bias)
        self._reset_parameters()

    def _reset_parameters(self):
        for lin in (self.q_proj, self.k_proj, self.v_proj, self.o_proj):
            nn.init.xavier_uniform_(lin.weight)
            if lin.bias is not None:
                nn.init.zeros_(lin.bias)

    def forward(self, x: torch.Tensor, kv: Optional[torch.Tensor] = None) -> torch.Tensor:
        B, S, D = x.shape
        kv = kv if kv is not None else x
        q = self.q_proj(x).view(B, S, self.n_heads, self.head_dim).transpose(1, 2)
        k = self.k_proj(kv).view(B, S, self.n_kv_heads, self.head_dim).transpose(1, 2)
        v = self.v_proj(kv).view(B, S, self.n_kv_heads, self.head_dim).transpose(1, 2)
        out = cron_root_attention_v14(q, k, v, kv_groups=self.kv_groups)
        out = out.permute(0, 2, 1, 3).reshape(B, S, D)
        return self.drop(self.o_proj(out))


class CronRootMultiheadAttention(nn.Module):
    """Drop-in for nn.MultiheadAttention (self-attention, always causal).

    forward(query, key, value, ...) -> (out, None); masks are ignored, as in
    the reference (module.py:186-247).
    """

    def __init__(self, embed_dim: int, num_heads: int, dropout: float = 0.0, bias: bool = True,
                 batch_first: bool = True):
        super().__init__()
        self.embed_dim = embed_dim
        self.num_heads = num_heads
        self.head_dim = embed_dim // num_heads
        self.dropout = dropout
        self.batch_first = batch_first
        assert embed_dim % num_heads == 0, "embed_dim must be divisible by num_heads"
        self.in_proj_weight = nn.Parameter(torch.empty(3 * embed_dim, embed_dim))
        if bias:
            self.in_proj_bias = nn.Parameter(torch.empty(3 * embed_dim))
        else:
            self.register_parameter("in_proj_bias", None)
        self.out_proj = nn.Linear(embed_dim, embed_dim, bias=bias)
        self.drop = nn.Dropout(dropout) if dropout > 0 else nn.Identity()
        self._reset_parameters()

    def _reset_parameters(self):
        nn.init.xavier_uniform_(self.in_proj_weight)
        if self.in_proj_bias is not None:
            nn.init.zeros_(self.in_proj_bias)
        nn.init.xavier_uniform_(self.out_proj.weight)
        if self.out_proj.bias is not None:
            nn.init.zeros_(self.out_proj.bias)

    def forward(self, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                key_padding_mask: Optional[torch.Tensor] = None, need_weights: bool = False,
                attn_mask: Optional[torch.Tensor] = None, average_attn_weights: bool = True,
                is_causal: bool = True) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
        if not self.batch_first:
            query, key, value = query.transpose(0, 1), key.transpose(0, 1), value.transpose(0, 1)
        B, S, D = query.shape
        assert query is key and key is value, "Cross-attention not yet supported"
        qkv = F.linear(query, self.in_proj_weight, self.in_proj_bias)
        qkv = qkv.view(B, S, 3, self.num_heads, self.head_dim).permute(2, 0, 3, 1, 4)
        out = cron_root_attention_v14(qkv[0], qkv[1], qkv[2])
        out = out.permute(0, 2, 1, 3).reshape(B, S, D)
        out = self.drop(self.out_proj(out))
        if not self.batch_first:
            out = out.transpose(0, 1)
        return out, None
