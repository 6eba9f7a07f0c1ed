"""Multi-GPU execution: one process per GPU, torch.distributed for plumbing.

Two ways to spread the work, matching how the attention decomposes:

* Head / batch sharding (``shard_units``): every (b, h) pair is independent,
  so each rank runs the ordinary op on its slice -- no collective at all.

* Sequence split (``seq_parallel_forward``): one very long sequence is cut
  into W-block-aligned query ranges, one per rank.  A rank's queries need
    - the local window: its own K/V rows plus the last W - 1 rows of the
      previous rank (the halo), and
    - the global rows (strided key + relay tokens of every W-block) of the
      WHOLE sequence.
  Each rank builds the global rows of its own blocks, then one all-gather
  (NCCL over NVLink on GPUs) assembles the full list in every rank's memory;
  the halo rows go point to point to the next rank only, which reads them
  (with its own first rows) from a small edge copy.  Everything lands in
  local HBM before the forward kernel reads it.

Reference: the reference package is single-GPU (no collectives); the
decomposition follows the attention's own structure (geom.cuh in libcra).
"""
from __future__ import annotations

import functools

import ctypes
import math
from typing import Optional, Sequence, Tuple

import numpy as np
import torch
import torch.distributed as dist


def window(seq_len: int) -> int:
    """W = ceil(sqrt(seq_len)) (reference core.py:3479)."""
    w = int(math.ceil(math.sqrt(seq_len)))
    while (w - 1) * (w - 1) >= seq_len:
        w -= 1
    while w * w < seq_len:
        w += 1
    return w


def shard_units(batch: int, heads: int, world: int, rank: int) -> Sequence[Tuple[int, int, int]]:
    """(b, h0, h1) slices of the batch x heads grid owned by ``rank``: heads
    split evenly when heads % world == 0, otherwise the flattened (b, h) grid
    is split into near-equal contiguous runs."""
    if heads % world == 0:
        per = heads // world
        return [(b, rank * per, (rank + 1) * per) for b in range(batch)]
    total = batch * heads
    u0, u1 = total * rank // world, total * (rank + 1) // world
    out = []
    u = u0
    while u < u1:
        b, h = divmod(u, heads)
        h1 = min(heads, h + (u1 - u))
        out.append((b, h, h1))
        u += h1 - h
    return out


@functools.lru_cache(maxsize=64)
def _shard_bounds(seq_len: int, world: int, top_k: int = 2) -> Tuple[int, ...]:
    """Block indices where each rank's W-blocks start (plus the end), chosen so
    that every rank gets about the same attention work: a query m attends
    min(m + 1, W) local keys and gcount(m) = R * floor(ls / W) + [ls % W != 0]
    global rows (ls = max(m - W + 1, 0), R = 1 + top_k with the relay, else
    1), so
    later queries cost more and equal row counts would leave the last rank
    with the most work."""
    W = window(seq_len)
    nb = (seq_len + W - 1) // W
    if nb < world:
        raise ValueError(f"{nb} W-blocks cannot be split across {world} ranks")
    R = 1 + top_k if seq_len > 2048 else 1
    m = np.arange(seq_len, dtype=np.int64)
    ls = np.maximum(m - W + 1, 0)
    work = np.minimum(m + 1, W) + R * (ls // W) + (ls % W != 0)
    per_block = np.add.reduceat(work, np.arange(0, seq_len, W))
    cum = np.concatenate([[0], np.cumsum(per_block)]).astype(np.float64)
    bounds = [0]
    for r in range(1, world):
        target = cum[-1] * r / world
        blk = int(np.searchsorted(cum, target))  # first block boundary at or past the target
        blk = min(max(blk, bounds[-1] + 1), nb - (world - r))  # every rank keeps >= 1 block
        bounds.append(blk)
    bounds.append(nb)
    return tuple(bounds)


def seq_shard(seq_len: int, world: int, rank: int, top_k: int = 2) -> Tuple[int, int]:
    """Query range [begin, end) of ``rank`` for a sequence split across
    ``world`` ranks: block-aligned, contiguous, with about equal attention
    work per rank (``_shard_bounds``) for ``top_k`` relay tokens per block."""
    W = window(seq_len)
    bounds = _shard_bounds(seq_len, world, top_k)
    return bounds[rank] * W, min(bounds[rank + 1] * W, seq_len)


class LibcraShardOps:
    """The two compute steps of the sequence split, on this GPU (libcra)."""

    def relay_build_shard(self, k, v, seq_len, row_begin, use_relay, top_k, relay_log_scale, with_src=False):
        from . import _lib
        from .core import _dtype_code, _stream_ptr
        L = _lib.lib()
        B, Hkv, rows, D = k.shape
        W = window(seq_len)
        R = 1 + top_k if use_relay else 1
        nblk = (rows + W - 1) // W
        gk = torch.empty(B, Hkv, nblk * R, D, device=k.device, dtype=k.dtype)
        gv = torch.empty_like(gk)
        gsrc = torch.empty(B, Hkv, nblk, top_k, device=k.device, dtype=torch.int32)
        alpha = None
        if relay_log_scale is not None and use_relay:
            alpha = relay_log_scale.detach().to(device=k.device, dtype=torch.float32).contiguous()
            if alpha.numel() != Hkv:
                raise ValueError(f"relay_log_scale must have H_kv = {Hkv} elements, got {alpha.numel()}")
        with torch.cuda.device(k.device):
            _lib.check(L.cra_relay_build_shard(k.data_ptr(), v.data_ptr(), _lib.strides3(k), _lib.strides3(v), B, Hkv,
                                               seq_len, row_begin, rows, D, _dtype_code(k.dtype), int(use_relay),
                                               top_k, alpha.data_ptr() if alpha is not None else None,
                                               gk.data_ptr(), gv.data_ptr(), gsrc.data_ptr(),
                                               _stream_ptr(k.device)), "cra_relay_build_shard")
        return (gk, gv, gsrc) if with_src else (gk, gv)

    def forward_shard(self, q, k, v, gk, gv, seq_len, q_begin, kv_begin, use_relay, top_k, edge=None,
                      return_lse=False):
        """Forward of one shard.  ``edge`` = (k_edge, v_edge, edge_begin): a
        small copy of the halo rows and the shard's first rows; then k / v
        are the shard's own rows (kv_begin = q_begin)."""
        from . import _lib
        from .core import _dtype_code, _err_word, _stream_ptr
        L = _lib.lib()
        B, H, q_len, D = q.shape
        Hkv, kv_len = k.shape[1], k.shape[2]
        o = torch.empty_like(q)
        lse = torch.empty(B, H, q_len, device=q.device, dtype=torch.float32)
        st = _lib.strides3
        if edge is not None:
            ke, ve, e0 = edge
            eargs = (ke.data_ptr(), ve.data_ptr(), st(ke), st(ve), e0, ke.shape[2])
        else:
            eargs = (None, None, None, None, 0, 0)
        with torch.cuda.device(q.device):
            _lib.check(L.cra_fwd_shard(q.data_ptr(), k.data_ptr(), v.data_ptr(), gk.data_ptr(), gv.data_ptr(),
                                       st(q), st(k), st(v), B, H, Hkv, seq_len, q_begin, q_len, kv_begin, kv_len,
                                       *eargs, D, _dtype_code(q.dtype), int(use_relay), top_k,
                                       ctypes.c_float(D ** -0.5), o.data_ptr(), st(o), lse.data_ptr(),
                                       _err_word(q.device).data_ptr(), _stream_ptr(q.device)), "cra_fwd_shard")
        return (o, lse) if return_lse else o

    def backward_shard(self, q, k, v, o, do, lse, gk, gv, gsrc, seq_len, q_begin, use_relay, top_k, edge,
                       relay_log_scale, all_reduce):
        """Backward of one shard: phase 1 (dG of this shard's queries),
        ``all_reduce`` sums dG over the shards in place, phase 2 (dq, dk, dv
        and the halo keys' dk / dv).  Returns dq, dk, dv, dk_halo, dv_halo
        (None for the first shard) and d(relay_log_scale) (None without)."""
        dgk, dgv, ws = self.backward_global(q, o, do, lse, gk, gv, seq_len, q_begin, use_relay, top_k)
        all_reduce(dgk)
        all_reduce(dgv)
        return self.backward_local(q, k, v, do, gk, gv, gsrc, dgk, dgv, ws, seq_len, q_begin, use_relay, top_k, edge,
                                   relay_log_scale)

    def backward_global(self, q, o, do, lse, gk, gv, seq_len, q_begin, use_relay, top_k):
        """Phase 1: fp32 dG_k, dG_v of every global row from this shard's
        queries, and the workspace phase 2 reuses."""
        from . import _lib
        from .core import _dtype_code, _err_word, _stream_ptr
        L = _lib.lib()
        B, H, q_len, D = q.shape
        Hkv, NG = gk.shape[1], gk.shape[2]
        st = _lib.strides3
        dev = q.device
        ws_b = L.cra_bwd_shard_workspace_bytes(B, H, Hkv, seq_len, q_len, D, int(use_relay), top_k)
        ws = torch.empty(max(ws_b, 1), device=dev, dtype=torch.uint8)
        dgk = torch.empty(B, Hkv, NG, D, device=dev, dtype=torch.float32)
        dgv = torch.empty_like(dgk)
        with torch.cuda.device(dev):
            _lib.check(L.cra_bwd_shard_global(q.data_ptr(), o.data_ptr(), do.data_ptr(), lse.data_ptr(), gk.data_ptr(),
                                              gv.data_ptr(), st(q), st(o), st(do), B, H, Hkv, seq_len, q_begin, q_len,
                                              D, _dtype_code(q.dtype), int(use_relay), top_k,
                                              ctypes.c_float(D ** -0.5), dgk.data_ptr(), dgv.data_ptr(),
                                              ws.data_ptr(), ws_b, _err_word(dev).data_ptr(), _stream_ptr(dev)),
                       "cra_bwd_shard_global")
        return dgk, dgv, ws

    def backward_local(self, q, k, v, do, gk, gv, gsrc, dgk, dgv, ws, seq_len, q_begin, use_relay, top_k, edge,
                       relay_log_scale):
        """Phase 2 (after dG was summed over the shards)."""
        from . import _lib
        from .core import _dtype_code, _err_word, _stream_ptr
        L = _lib.lib()
        B, H, q_len, D = q.shape
        Hkv = k.shape[1]
        st = _lib.strides3
        dev = q.device
        dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
        alpha = None
        if relay_log_scale is not None and use_relay:
            alpha = relay_log_scale.detach().to(device=dev, dtype=torch.float32).contiguous()
        dalpha = torch.zeros(Hkv, device=dev, dtype=torch.float32) if alpha is not None else None
        W = window(seq_len)
        n_halo = min(W - 1, q_begin)
        if q_begin > 0:
            ke, ve, e0 = edge
            dkh = torch.empty(B, Hkv, n_halo, D, device=dev, dtype=k.dtype)
            dvh = torch.empty_like(dkh)
            eargs = (ke.data_ptr(), ve.data_ptr(), st(ke), st(ve), e0, ke.shape[2])
            hargs = (dkh.data_ptr(), dvh.data_ptr())
            hst = (st(dkh), st(dvh))
        else:
            dkh = dvh = None
            eargs = (None, None, None, None, 0, 0)
            hargs = (None, None)
            hst = (None, None)
        with torch.cuda.device(dev):
            _lib.check(L.cra_bwd_shard_local(q.data_ptr(), k.data_ptr(), v.data_ptr(), do.data_ptr(), gk.data_ptr(),
                                             gv.data_ptr(), gsrc.data_ptr(), st(q), st(k), st(v), st(do), *eargs, B, H,
                                             Hkv, seq_len, q_begin, q_len, D, _dtype_code(q.dtype), int(use_relay),
                                             top_k, ctypes.c_float(D ** -0.5),
                                             alpha.data_ptr() if alpha is not None else None, dgk.data_ptr(),
                                             dgv.data_ptr(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), *hargs,
                                             st(dq), st(dk), st(dv), *hst,
                                             dalpha.data_ptr() if dalpha is not None else None, ws.data_ptr(),
                                             ws.numel(), _err_word(dev).data_ptr(), _stream_ptr(dev)),
                       "cra_bwd_shard_local")
        return dq, dk, dv, dkh, dvh, dalpha


def _all_gather_padded(x: torch.Tensor, dim: int, sizes: Sequence[int], group) -> torch.Tensor:
    """Concatenate, along ``dim``, every rank's ``x`` (rank r contributes
    sizes[r] rows); pads to the largest size for the collective."""
    if len(sizes) == 1:  # one rank: nothing to exchange
        return x.narrow(dim, 0, sizes[0])
    mx = max(sizes)
    pad = mx - x.shape[dim]
    if pad:
        shape = list(x.shape)
        shape[dim] = pad
        x = torch.cat([x, x.new_zeros(shape)], dim=dim)
    x = x.contiguous()
    parts = [torch.empty_like(x) for _ in sizes]
    dist.all_gather(parts, x, group=group)
    return torch.cat([p.narrow(dim, 0, s) for p, s in zip(parts, sizes)], dim=dim)


def _world(group):
    if group is None and not (dist.is_available() and dist.is_initialized()):
        return 1, 0  # a single process: the whole sequence, no exchange
    return dist.get_world_size(group), dist.get_rank(group)


def _peer(group, rank):
    return rank if group is None else dist.get_global_rank(group, rank)


def _seq_forward(q, k, v, seq_len, group, relay_top_k, relay_log_scale, ops, keep_state):
    world, rank = _world(group)
    ops = ops or LibcraShardOps()
    begin, end = seq_shard(seq_len, world, rank, relay_top_k)
    if q.shape[2] != end - begin or k.shape[2] != end - begin:
        raise ValueError(f"rank {rank} owns rows [{begin}, {end}) but got {q.shape[2]}")
    W = window(seq_len)
    use_relay = seq_len > 2048  # reference core.py:2832,3507
    R = 1 + relay_top_k if use_relay else 1
    # 1) global rows of this rank's blocks, then the whole list everywhere
    gk, gv, gsrc = ops.relay_build_shard(k, v, seq_len, begin, use_relay, relay_top_k, relay_log_scale, with_src=True)
    bounds = [seq_shard(seq_len, world, r, relay_top_k) for r in range(world)]
    rows = [((e - b + W - 1) // W) * R for b, e in bounds]
    gk = _all_gather_padded(gk, 2, rows, group)
    gv = _all_gather_padded(gv, 2, rows, group)
    if keep_state:  # the backward's fold-in reads every block's relay sources
        gsrc = _all_gather_padded(gsrc, 2, [(e - b + W - 1) // W for b, e in bounds], group)
    # 2) halo: the last W - 1 K/V rows of the previous rank, sent to the next
    # rank only (point to point); the receiver builds a small edge copy --
    # halo rows followed by its own first W + 256 rows -- which the query
    # tiles whose window reaches into the halo read, so the shard's own K / V
    # are used in place (no copy of the whole shard)
    halo = W - 1
    n_in = 0
    recv = None
    if world > 1:
        ops_p2p = []
        if rank + 1 < world:
            tail = torch.cat([k[:, :, max(0, k.shape[2] - halo):], v[:, :, max(0, v.shape[2] - halo):]], dim=1)
            ops_p2p.append(dist.P2POp(dist.isend, tail.contiguous(), _peer(group, rank + 1), group))
        if rank > 0:
            prev_b, prev_e = bounds[rank - 1]
            n_in = min(halo, prev_e - prev_b)
            recv = k.new_empty(k.shape[0], 2 * k.shape[1], n_in, k.shape[3])
            ops_p2p.append(dist.P2POp(dist.irecv, recv, _peer(group, rank - 1), group))
        for req in dist.batch_isend_irecv(ops_p2p):
            req.wait()
    qc, kc, vc = q.contiguous(), k.contiguous(), v.contiguous()
    gk, gv = gk.contiguous(), gv.contiguous()
    edge = None
    if rank > 0 and n_in > 0:
        Hkv = k.shape[1]
        X = min(W + 256, k.shape[2])
        ke = torch.cat([recv[:, :Hkv], k[:, :, :X]], dim=2).contiguous()
        ve = torch.cat([recv[:, Hkv:], v[:, :, :X]], dim=2).contiguous()
        edge = (ke, ve, begin - n_in)
        o, lse = ops.forward_shard(qc, kc, vc, gk, gv, seq_len, begin, begin, use_relay, relay_top_k, edge=edge,
                                   return_lse=True)
    else:
        o, lse = ops.forward_shard(qc, kc, vc, gk, gv, seq_len, begin, 0 if rank == 0 else begin, use_relay,
                                   relay_top_k, return_lse=True)
    state = None
    if keep_state:
        state = dict(world=world, rank=rank, begin=begin, use_relay=use_relay, gk=gk, gv=gv,
                     gsrc=gsrc.contiguous(), edge=edge, lse=lse, q=qc, k=kc, v=vc, ops=ops)
    return o, state


@torch.no_grad()
def seq_parallel_forward(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, seq_len: int,
                         group=None, relay_top_k: int = 2, relay_log_scale: Optional[torch.Tensor] = None,
                         ops=None) -> torch.Tensor:
    """Forward of one sequence split across the ranks of ``group``.

    q, k, v: this rank's rows, [B, H, end - begin, D] with (begin, end) =
    seq_shard(seq_len, world, rank).  Returns this rank's output rows.
    Collectives: one all-gather (global rows) and one neighbour send/recv
    (halo rows); no data-dependent host synchronisation.  Without an
    initialized process group (and no ``group`` given) it runs as a single
    rank.
    """
    return _seq_forward(q, k, v, seq_len, group, relay_top_k, relay_log_scale, ops, False)[0]


class _SeqParallelFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, seq_len, group, relay_top_k, relay_log_scale, ops):
        o, st = _seq_forward(q, k, v, seq_len, group, relay_top_k, relay_log_scale, ops, True)
        ctx.st = st
        ctx.o = o
        ctx.meta = (seq_len, group, relay_top_k, relay_log_scale)
        return o

    @staticmethod
    def backward(ctx, do):
        st, o = ctx.st, ctx.o
        seq_len, group, top_k, alpha = ctx.meta
        world, rank = st["world"], st["rank"]

        def all_reduce(t):
            if world > 1:
                dist.all_reduce(t, group=group)

        dq, dk, dv, dkh, dvh, dalpha = st["ops"].backward_shard(
            st["q"], st["k"], st["v"], o, do.contiguous(), st["lse"], st["gk"], st["gv"], st["gsrc"], seq_len,
            st["begin"], st["use_relay"], top_k, st["edge"], alpha, all_reduce)
        # the halo keys' gradients go back to the previous rank, which adds
        # them to its last rows
        if world > 1:
            W = window(seq_len)
            ops_p2p = []
            recv = None
            if rank > 0:
                ops_p2p.append(dist.P2POp(dist.isend, torch.cat([dkh, dvh], dim=1).contiguous(),
                                          _peer(group, rank - 1), group))
            if rank + 1 < world:
                n = min(W - 1, dk.shape[2])
                recv = dk.new_empty(dk.shape[0], 2 * dk.shape[1], n, dk.shape[3])
                ops_p2p.append(dist.P2POp(dist.irecv, recv, _peer(group, rank + 1), group))
            for req in dist.batch_isend_irecv(ops_p2p):
                req.wait()
            if recv is not None:
                n, Hkv = recv.shape[2], dk.shape[1]
                dk[:, :, dk.shape[2] - n:] += recv[:, :Hkv]
                dv[:, :, dv.shape[2] - n:] += recv[:, Hkv:]
        d_alpha = None
        if alpha is not None:  # the summed scale gradient, reported by rank 0 only
            d_alpha = dalpha if (dalpha is not None and rank == 0) else torch.zeros_like(alpha, dtype=torch.float32)
        ctx.st = ctx.o = None
        return dq, dk, dv, None, None, None, d_alpha, None


def seq_parallel_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, seq_len: int, group=None,
                           relay_top_k: int = 2, relay_log_scale: Optional[torch.Tensor] = None,
                           ops=None) -> torch.Tensor:
    """Differentiable sequence-split attention: the forward of
    ``seq_parallel_forward`` plus a backward in which every rank computes the
    gradients of its own queries -- dG of the global rows (summed over the
    ranks with one all-reduce, then folded into the keys of each rank's own
    blocks), dq, dk / dv of its keys, and the contributions to the previous
    rank's last W - 1 keys, sent back point to point.  The gradient of
    ``relay_log_scale`` is the total on rank 0 and zero elsewhere, so a sum
    over ranks (as data-parallel gradient averaging does, up to its scale)
    counts it once."""
    return _SeqParallelFunction.apply(q, k, v, seq_len, group, relay_top_k, relay_log_scale, ops)
