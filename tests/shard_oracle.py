"""CPU stand-ins for the two compute steps of the sequence split (test
infrastructure): built from the oracle's definitions so that the gloo tests
check the host-side exchange logic of cron_root_attention.parallel."""
import math

import torch

from oracle import cra_oracle as O


def gcount(m, W, R):
    ls = max(m - W + 1, 0)
    return R * (ls // W) + (1 if ls % W else 0)


class OracleShardOps:
    def relay_build_shard(self, k, v, seq_len, row_begin, use_relay, top_k, relay_log_scale):
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
        return torch.cat(out_k, 2), torch.cat(out_v, 2)

    def forward_shard(self, q, k, v, gk, gv, seq_len, q_begin, kv_begin, use_relay, top_k, edge=None):
        if edge is not None:  # halo rows from the edge copy in front of the shard's own rows
            ke, ve, e0 = edge
            k = torch.cat([ke[:, :, :kv_begin - e0], k], 2)
            v = torch.cat([ve[:, :, :kv_begin - e0], v], 2)
            kv_begin = e0
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
        p = torch.softmax(s, -1)
        return p[..., :k.shape[2]] @ v + p[..., k.shape[2]:] @ gv
