"""CPU stand-ins for the compute steps of the sequence split (test
infrastructure): built from the oracle's definitions so that the gloo tests
check the host-side exchange logic of cron_root_attention.parallel --
forward (global rows, halo) and backward (summed global-row gradients,
halo gradients sent back)."""
import math

import torch

from oracle import cra_oracle as O


def gcount(m, W, R):
    ls = max(m - W + 1, 0)
    return R * (ls // W) + (1 if ls % W else 0)


class OracleShardOps:
    def relay_build_shard(self, k, v, seq_len, row_begin, use_relay, top_k, relay_log_scale, with_src=False):
        B, H, rows, D = k.shape
        W = O.window(seq_len)
        nblk = (rows + W - 1) // W
        out_k, out_v = [], []
        ridx = O.relay_select(k, W, top_k) if use_relay else None  # local positions
        for r in range(nblk):
            idx = [torch.full((B, H), r * W, dtype=torch.long)]
            if use_relay:
                idx += [ridx[:, :, r, t] for t in range(top_k)]
            for i in idx:
                out_k.append(torch.gather(k, 2, i.view(B, H, 1, 1).expand(B, H, 1, D)))
                out_v.append(torch.gather(v, 2, i.view(B, H, 1, 1).expand(B, H, 1, D)))
        gk, gv = torch.cat(out_k, 2), torch.cat(out_v, 2)
        if not with_src:
            return gk, gv
        src = (ridx + row_begin) if use_relay else torch.zeros(B, H, nblk, top_k, dtype=torch.long)
        return gk, gv, src

    @staticmethod
    def _attend(q, k, v, gk, gv, seq_len, q_begin, kv_begin, use_relay, top_k):
        B, H, n, D = q.shape
        W = O.window(seq_len)
        R = 1 + top_k if use_relay else 1
        m = torch.arange(q_begin, q_begin + n).view(-1, 1)
        ls = (m - W + 1).clamp(min=0)
        kpos = torch.arange(kv_begin, kv_begin + k.shape[2]).view(1, -1)
        lm = (kpos >= ls) & (kpos <= m)
        cnt = R * (ls // W) + (ls % W != 0).long()
        gm = torch.arange(gk.shape[2]).view(1, -1) < cnt
        s = torch.cat([(q @ k.transpose(-1, -2)).masked_fill(~lm, float("-inf")),
                       (q @ gk.transpose(-1, -2)).masked_fill(~gm, float("-inf"))], -1) / math.sqrt(D)
        lse = torch.logsumexp(s, -1)
        p = torch.softmax(s, -1)
        return p[..., :k.shape[2]] @ v + p[..., k.shape[2]:] @ gv, lse

    def forward_shard(self, q, k, v, gk, gv, seq_len, q_begin, kv_begin, use_relay, top_k, edge=None,
                      return_lse=False):
        if edge is not None:  # halo rows from the edge copy in front of the shard's own rows
            ke, ve, e0 = edge
            k = torch.cat([ke[:, :, :kv_begin - e0], k], 2)
            v = torch.cat([ve[:, :, :kv_begin - e0], v], 2)
            kv_begin = e0
        o, lse = self._attend(q, k, v, gk, gv, seq_len, q_begin, kv_begin, use_relay, top_k)
        return (o, lse) if return_lse else o

    def backward_shard(self, q, k, v, o, do, lse, gk, gv, gsrc, seq_len, q_begin, use_relay, top_k, edge,
                       relay_log_scale, all_reduce):
        W = O.window(seq_len)
        R = 1 + top_k if use_relay else 1
        n_h = min(W - 1, q_begin)
        with torch.enable_grad():  # called from inside an autograd backward
            leaf = lambda t: t.detach().clone().requires_grad_(True)
            qq, kk, vv, gkk, gvv = (leaf(t) for t in (q, k, v, gk, gv))
            if n_h > 0:
                ke, ve, e0 = edge
                kh, vh = leaf(ke[:, :, q_begin - n_h - e0:q_begin - e0]), leaf(ve[:, :, q_begin - n_h - e0:q_begin - e0])
                kx, vx = torch.cat([kh, kk], 2), torch.cat([vh, vv], 2)
            else:
                kh = vh = None
                kx, vx = kk, vv
            out, _ = self._attend(qq, kx, vx, gkk, gvv, seq_len, q_begin, q_begin - n_h, use_relay, top_k)
            (out * do).sum().backward()
        dgk, dgv = gkk.grad.clone(), gvv.grad.clone()
        all_reduce(dgk)
        all_reduce(dgv)
        dk, dv = kk.grad.clone(), vv.grad.clone()
        B, H, rows, D = k.shape
        for blk in range(q_begin // W, (q_begin + rows + W - 1) // W):  # this shard's blocks: fold in dG
            dk[:, :, blk * W - q_begin] += dgk[:, :, blk * R]
            dv[:, :, blk * W - q_begin] += dgv[:, :, blk * R]
            for t in range(R - 1):
                for b in range(B):
                    for h in range(H):
                        src = int(gsrc[b, h, blk, t]) - q_begin
                        dk[b, h, src] += dgk[b, h, blk * R + 1 + t]
                        dv[b, h, src] += dgv[b, h, blk * R + 1 + t]
        return (qq.grad, dk, dv, kh.grad if kh is not None else None, vh.grad if vh is not None else None, None)
