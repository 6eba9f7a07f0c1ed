"""CPU oracle for the causal 3-phase sqrt(N) attention (Cron Root Attention).

TEST INFRASTRUCTURE ONLY.  This module is the checker that the CUDA path is
compared against.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import it.
The shipped library never calls it and has no CPU fallback.

It restates, in plain torch CPU code (fp32 or fp64), the reference's own CPU
implementation ``cron_root_attention/cpu_reference.py:198-339``
(``cra_cpu_fast``), with the window the reference's GPU path uses
(``W = ceil(sqrt(S))``, ``cron_root_attention/core.py:3479``) and the GPU
path's relay switch (relay off for ``S <= 2048``, ``core.py:2832,3507``).
Pinning: ``tests/golden/make_golden.py`` ran the reference's ``cra_cpu_fast``
itself (with W forced to ceil(sqrt(S))) and stored its outputs; the tests
check this restatement against those fixtures.

The reference has no CPU backward.  ``forward_backward`` below is a
differentiable, out-of-place restatement of the same math (relay rows are
gathered by index, so their gradients land on the source tokens the way
``core.py:2767-2815`` scatters them; relay *selection* is a constant).  Its
forward is checked equal to the pinned forward, which is what pins it.

Semantics (one query m, ls = max(m - W + 1, 0)):
  * local keys j in [ls, m]                               core.py:993-994
  * strided keys j = sW with j < ls                        core.py:1059
  * relay token t of block r = t // TOP_K visible iff
    (r + 1) * W - 1 < ls                                   core.py:1115-1116
  * relay tokens = the TOP_K rows of block r with the largest ||k||^2,
    ties to the lower index (core.py:2685-2703), copied exactly
    (core.py:2715-2730), optionally scaled by exp(relay_log_scale[h])
    (core.py:3541-3544)
  * one softmax over the union, scale 1/sqrt(D); out = acc / l;
    lse = max + log(l)                                     core.py:1147-1158
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional

import torch

RELAY_THRESHOLD = 2048  # core.py:2832 -- relay is skipped for S <= 2048


def window(S: int) -> int:
    """W = ceil(sqrt(S)) as the reference GPU path computes it (core.py:3479)."""
    return int(math.ceil(math.sqrt(S)))


def relay_active(S: int) -> bool:
    """core.py:3507: ``skip_relay = S <= RELAY_THRESHOLD``."""
    return S > RELAY_THRESHOLD


def num_blocks(S: int, W: int) -> int:
    return (S + W - 1) // W


def relay_select(k: torch.Tensor, W: int, top_k: int) -> torch.Tensor:
    """Top-``top_k`` row indices per W-block by ||k||^2 (core.py:2630-2748).

    Norms are taken in float64 of the given values (exact for fp16/bf16
    inputs).  Ties go to the lower index, as the reference's strict ``>``
    insertion sort does (core.py:2685-2696).  Rows past S are never chosen
    unless the block has fewer valid rows than ``top_k``; then the block's
    first row repeats (core.py:2682 initialises the indices to 0).  Such a
    block is always the last one, which no query ever sees.

    Returns int64 absolute positions, shape [B, H, NB, top_k].
    """
    B, H, S, D = k.shape
    NB = num_blocks(S, W)
    pad = NB * W - S
    n = (k.double() ** 2).sum(-1)  # [B,H,S]
    if pad:
        n = torch.cat([n, torch.full((B, H, pad), -1.0, dtype=n.dtype)], dim=2)
    n = n.view(B, H, NB, W)
    # stable descending sort keeps the lower index first among equal norms
    order = torch.sort(n, dim=-1, descending=True, stable=True).indices[..., :top_k]
    if order.shape[-1] < top_k:  # W < top_k: repeat the first row index
        order = torch.cat([order, order[..., :1].expand(*order.shape[:-1], top_k - order.shape[-1])], -1)
    base = (torch.arange(NB) * W).view(1, 1, NB, 1)
    pos = order + base
    valid = pos < S
    pos = torch.where(valid, pos, base.expand_as(pos))
    return pos


@dataclass
class GlobalList:
    """Strided + relay key rows in the order the reference's ``cra_cpu_fast``
    concatenates them (cpu_reference.py:245-268): all strided rows, then the
    relay rows block by block."""

    idx: torch.Tensor       # [B,H,NG] int64 source positions
    is_relay: torch.Tensor  # [NG] bool
    visible_before: torch.Tensor  # [NG] int64: row visible iff this value < ls


def build_global_list(k: torch.Tensor, W: int, use_relay: bool, top_k: int,
                      relay_idx: Optional[torch.Tensor] = None) -> GlobalList:
    B, H, S, D = k.shape
    stride_pos = torch.arange(0, S, W)
    NS = stride_pos.numel()
    idx = stride_pos.view(1, 1, NS).expand(B, H, NS)
    vis = stride_pos.clone()                    # strided key sW visible iff sW < ls
    is_relay = torch.zeros(NS, dtype=torch.bool)
    if use_relay:
        NB = num_blocks(S, W)
        if relay_idx is None:
            relay_idx = relay_select(k, W, top_k)
        r_idx = relay_idx.reshape(B, H, NB * top_k)
        t = torch.arange(NB * top_k)
        r_vis = (t // top_k + 1) * W - 1        # block_end < ls  (core.py:1115)
        idx = torch.cat([idx, r_idx], dim=2)
        vis = torch.cat([vis, r_vis])
        is_relay = torch.cat([is_relay, torch.ones(NB * top_k, dtype=torch.bool)])
    return GlobalList(idx=idx.contiguous(), is_relay=is_relay, visible_before=vis)


def _gather_rows(x: torch.Tensor, idx: torch.Tensor) -> torch.Tensor:
    B, H, S, D = x.shape
    return torch.gather(x, 2, idx.unsqueeze(-1).expand(B, H, idx.shape[-1], D))


def forward(q, k, v, *, use_relay: Optional[bool] = None, top_k: int = 2,
            relay_log_scale: Optional[torch.Tensor] = None,
            relay_idx: Optional[torch.Tensor] = None, W: Optional[int] = None,
            chunk: int = 256, dtype=torch.float32, kv_groups: int = 1, rows=None,
            relay_dtype=None):
    """Forward restatement of cpu_reference.py:198-339 (``cra_cpu_fast``).

    ``rows=(r0, r1)`` computes only query rows [r0, r1) (others are left 0);
    each row depends only on its own keys, so those rows are exact.
    ``relay_dtype``: the reference keeps the scaled relay rows in the input
    dtype (``relay_k * exp(a).to(dtype)``, core.py:3541-3544); pass that dtype
    to round them the same way (the scale exp(a) is rounded too).

    Same chunked single-pass softmax: per chunk of ``chunk`` queries, scores
    against the local window and against the concatenated strided+relay rows,
    one max, exp, one sum, ``denom.clamp(min=1e-12)`` (cpu_reference.py:322-337).
    Returns (out, lse) in ``dtype``; lse is natural-log, [B,H,S].
    """
    q = q.to(dtype); k = k.to(dtype); v = v.to(dtype)
    B, Hq, S, D = q.shape
    if kv_groups > 1:  # cpu_reference.py:239-241
        k = k.repeat_interleave(kv_groups, dim=1)
        v = v.repeat_interleave(kv_groups, dim=1)
        if relay_idx is not None:
            relay_idx = relay_idx.repeat_interleave(kv_groups, dim=1)
        if relay_log_scale is not None:
            relay_log_scale = relay_log_scale.repeat_interleave(kv_groups)
    if W is None:
        W = window(S)
    if use_relay is None:
        use_relay = relay_active(S)
    scale = 1.0 / math.sqrt(D)
    gl = build_global_list(k, W, use_relay, top_k, relay_idx)
    Kg = _gather_rows(k, gl.idx)
    Vg = _gather_rows(v, gl.idx)
    if relay_log_scale is not None and use_relay:
        e = relay_log_scale.to(dtype).exp()
        if relay_dtype is not None:
            e = relay_log_scale.float().exp().to(relay_dtype)
        f = torch.where(gl.is_relay.view(1, 1, -1, 1), e.to(dtype).view(1, Hq, 1, 1),
                        torch.ones((), dtype=dtype))
        Kg = Kg * f
        Vg = Vg * f
        if relay_dtype is not None:
            Kg = Kg.to(relay_dtype).to(dtype)
            Vg = Vg.to(relay_dtype).to(dtype)
    out = torch.zeros(B, Hq, S, D, dtype=dtype)
    lse = torch.zeros(B, Hq, S, dtype=dtype)
    pos = torch.arange(S)
    r0, r1 = rows if rows is not None else (0, S)
    for q0 in range(r0, r1, chunk):
        q1 = min(q0 + chunk, r1)
        qc = q[:, :, q0:q1]
        w0 = max(0, q0 - W + 1)
        Kw, Vw = k[:, :, w0:q1], v[:, :, w0:q1]
        qp = pos[q0:q1].view(-1, 1)
        kp = pos[w0:q1].view(1, -1)
        ls = (qp - W + 1).clamp(min=0)
        m_l = (kp <= qp) & (kp >= qp - W + 1)
        m_g = gl.visible_before.view(1, -1) < ls
        s_l = torch.matmul(qc, Kw.transpose(-1, -2)) * scale
        s_g = torch.matmul(qc, Kg.transpose(-1, -2)) * scale
        s_l = s_l.masked_fill(~m_l, float("-inf"))
        s_g = s_g.masked_fill(~m_g, float("-inf"))
        mx = torch.maximum(s_l.amax(-1), s_g.amax(-1)).unsqueeze(-1)
        e_l = (s_l - mx).exp()
        e_g = (s_g - mx).exp()
        den = (e_l.sum(-1) + e_g.sum(-1)).clamp(min=1e-12)
        o = torch.matmul(e_l, Vw) + torch.matmul(e_g, Vg)
        out[:, :, q0:q1] = o / den.unsqueeze(-1)
        lse[:, :, q0:q1] = mx.squeeze(-1) + den.log()
    return out, lse


def forward_backward(q, k, v, do, *, use_relay: Optional[bool] = None, top_k: int = 2,
                     relay_log_scale: Optional[torch.Tensor] = None,
                     relay_idx: Optional[torch.Tensor] = None, W: Optional[int] = None,
                     chunk: int = 256, dtype=torch.float64, kv_groups: int = 1, rows=None,
                     relay_dtype=None):
    """Differentiable restatement; returns (out, dq, dk, dv, d_relay_log_scale).

    ``rows=(r0, r1)`` restricts the loss to query rows [r0, r1): dq of those
    rows is then exact (dk / dv only receive those rows' contributions).

    Autograd through gathered relay rows sends each relay row's gradient to
    its source token (what core.py:2767-2815 does on the GPU).  The relay
    scale is chained correctly: d(source) = exp(alpha) * d(relay row) and
    d(alpha) = sum(d(relay row) * relay row).  (The reference's GPU backward
    skips the exp(alpha) factor on the source gradient, core.py:3275-3282;
    with relay_log_scale=None the two agree.)
    """
    q = q.detach().to(dtype).requires_grad_(True)
    k = k.detach().to(dtype).requires_grad_(True)
    v = v.detach().to(dtype).requires_grad_(True)
    alpha = None
    if relay_log_scale is not None:
        alpha = relay_log_scale.detach().to(dtype).requires_grad_(True)
    B, Hq, S, D = q.shape
    kk, vv = k, v
    if kv_groups > 1:
        kk = k.repeat_interleave(kv_groups, dim=1)
        vv = v.repeat_interleave(kv_groups, dim=1)
        if relay_idx is not None:
            relay_idx = relay_idx.repeat_interleave(kv_groups, dim=1)
    al = alpha.repeat_interleave(kv_groups) if (alpha is not None and kv_groups > 1) else alpha
    if W is None:
        W = window(S)
    if use_relay is None:
        use_relay = relay_active(S)
    scale = 1.0 / math.sqrt(D)
    gl = build_global_list(kk.detach(), W, use_relay, top_k, relay_idx)
    Kg = _gather_rows(kk, gl.idx)
    Vg = _gather_rows(vv, gl.idx)
    if al is not None and use_relay:
        e = al.exp()
        if relay_dtype is not None:  # value rounded as the reference does; gradient straight through
            e = e + (e.detach().float().to(relay_dtype).to(dtype) - e.detach())
        f = torch.where(gl.is_relay.view(1, 1, -1, 1), e.view(1, Hq, 1, 1), torch.ones((), dtype=dtype))
        Kg = Kg * f
        Vg = Vg * f
        if relay_dtype is not None:
            Kg = Kg + (Kg.detach().float().to(relay_dtype).to(dtype) - Kg.detach())
            Vg = Vg + (Vg.detach().float().to(relay_dtype).to(dtype) - Vg.detach())
    pos = torch.arange(S)
    outs = []
    r0, r1 = rows if rows is not None else (0, S)
    for q0 in range(r0, r1, chunk):
        q1 = min(q0 + chunk, r1)
        qc = q[:, :, q0:q1]
        w0 = max(0, q0 - W + 1)
        qp = pos[q0:q1].view(-1, 1)
        kp = pos[w0:q1].view(1, -1)
        ls = (qp - W + 1).clamp(min=0)
        m_l = (kp <= qp) & (kp >= qp - W + 1)
        m_g = gl.visible_before.view(1, -1) < ls
        s_l = (torch.matmul(qc, kk[:, :, w0:q1].transpose(-1, -2)) * scale).masked_fill(~m_l, float("-inf"))
        s_g = (torch.matmul(qc, Kg.transpose(-1, -2)) * scale).masked_fill(~m_g, float("-inf"))
        p = torch.softmax(torch.cat([s_l, s_g], dim=-1), dim=-1)
        nl = s_l.shape[-1]
        outs.append(torch.matmul(p[..., :nl], vv[:, :, w0:q1]) + torch.matmul(p[..., nl:], Vg))
    out = torch.cat(outs, dim=2)
    grads = torch.autograd.grad(out, [q, k, v] + ([alpha] if alpha is not None else []),
                                grad_outputs=do.to(dtype)[:, :, r0:r1], allow_unused=True)
    dq, dk, dv = (g if g is not None else torch.zeros_like(t) for g, t in zip(grads[:3], (q, k, v)))
    da = grads[3] if alpha is not None else None
    if da is None and alpha is not None:
        da = torch.zeros_like(alpha)
    return out.detach(), dq, dk, dv, da


def dense_forward(q, k, v, *, use_relay=None, top_k=2, W=None, dtype=torch.float64):
    """Second, independent statement of the mask as one dense [S,S+NG] matrix.
    Small S only; used to cross-check ``forward``."""
    q = q.to(dtype); k = k.to(dtype); v = v.to(dtype)
    B, H, S, D = q.shape
    W = window(S) if W is None else W
    use_relay = relay_active(S) if use_relay is None else use_relay
    m = torch.arange(S).view(-1, 1)
    j = torch.arange(S).view(1, -1)
    ls = (m - W + 1).clamp(min=0)
    local = (j >= ls) & (j <= m)
    strided = (j % W == 0) & (j < ls)
    mask = local | strided  # strided keys never fall inside the local window
    scores = torch.matmul(q, k.transpose(-1, -2)) / math.sqrt(D)
    scores = scores.masked_fill(~mask, float("-inf"))
    cols = [scores]
    vals = [v]
    if use_relay:
        ridx = relay_select(k, W, top_k)  # [B,H,NB,K]
        NB = ridx.shape[2]
        r = ridx.reshape(B, H, NB * top_k)
        Kr = _gather_rows(k, r)
        Vr = _gather_rows(v, r)
        blk = torch.arange(NB * top_k) // top_k
        vis = ((blk + 1) * W - 1).view(1, -1) < ls
        sr = (torch.matmul(q, Kr.transpose(-1, -2)) / math.sqrt(D)).masked_fill(~vis, float("-inf"))
        cols.append(sr)
        vals.append(Vr)
    p = torch.softmax(torch.cat(cols, -1), -1)
    return torch.matmul(p, torch.cat(vals, 2))


def visible_pairs(S: int, W: Optional[int] = None, use_relay: Optional[bool] = None,
                  top_k: int = 2) -> int:
    """Exact count of visible (query, key) pairs per (b, h): local + strided +
    relay (relay counted top_k per visible block).  Used for FLOP accounting."""
    W = window(S) if W is None else W
    use_relay = relay_active(S) if use_relay is None else use_relay
    m = torch.arange(S, dtype=torch.int64)
    ls = (m - W + 1).clamp(min=0)
    local = (m - ls + 1).sum().item()
    strided = ((ls + W - 1) // W).sum().item()
    relay = (top_k * (ls // W)).sum().item() if use_relay else 0
    return int(local + strided + relay)
