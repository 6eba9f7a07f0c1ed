"""Model-quality check: train the same small causal transformer with this
package's attention and with dense causal attention (PyTorch SDPA) on
synthetic long-range recall tasks, and compare held-out token accuracy.

    python -m cron_root_attention.quality --task mqar --seq 4096 --steps 400

Covers what the reference's examples/bench_model_quality.py measures (it
trains small models on multi-query associative recall and selective copy);
the tasks are generated here, vectorised on the device:

* ``mqar``: n_kv (key, value) pairs, filler tokens, a separator, then
  n_queries keys whose values must be recalled.  Only the answer positions
  are scored.
* ``copy``: n_copy content tokens interleaved with a marker, filler, a
  separator, then the content tokens again, each predicted from the first
  copy.
* ``copy_near``: the same with the filler first, so the first copy sits in
  the local window of the recall positions: the sparse pattern sees all it
  needs there and should train like dense attention.

The sparse pattern sees every key through the local window only within
sqrt(S) tokens; earlier keys reach a query through the strided keys and the
two relay tokens per block, so recall far back is the interesting case.
"""
from __future__ import annotations

import argparse
import json
import math
import time
from typing import Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

N_FILL = 16  # filler vocabulary, disjoint from every scored token


def make_mqar(n: int, seq_len: int, n_kv: int, n_queries: int, gen: torch.Generator,
              device) -> Tuple[torch.Tensor, torch.Tensor, int]:
    """Returns (tokens [n, seq_len], targets [n, seq_len] with -100 where not
    scored, vocabulary size).  Tokens: 0 separator, 1 query marker, keys
    [2, 2 + n_kv), values [2 + n_kv, 2 + 2 n_kv), filler after those (the
    filler never repeats a key, so the pair region alone answers a query)."""
    k0, v0, f0 = 2, 2 + n_kv, 2 + 2 * n_kv
    vocab = f0 + N_FILL
    fill = seq_len - 2 * n_kv - 1 - 2 * n_queries
    if fill < 0:
        raise ValueError(f"seq_len {seq_len} too short for {n_kv} pairs and {n_queries} queries")
    keys = torch.argsort(torch.rand(n, n_kv, generator=gen, device=device), dim=1)
    vals = torch.randint(0, n_kv, (n, n_kv), generator=gen, device=device)
    x = torch.randint(f0, vocab, (n, seq_len), generator=gen, device=device)
    tgt = torch.full((n, seq_len), -100, dtype=torch.long, device=device)
    x[:, 0:2 * n_kv:2] = k0 + keys
    x[:, 1:2 * n_kv:2] = v0 + vals
    sep = 2 * n_kv + fill
    x[:, sep] = 0
    pick = torch.argsort(torch.rand(n, n_kv, generator=gen, device=device), dim=1)[:, :n_queries]
    qkeys = torch.gather(keys, 1, pick)
    qvals = torch.gather(vals, 1, pick)
    qpos = sep + 1 + 2 * torch.arange(n_queries, device=device)
    x[:, qpos] = k0 + qkeys
    x[:, qpos + 1] = 1
    tgt[:, qpos + 1] = v0 + qvals
    return x, tgt, vocab


def make_copy(n: int, seq_len: int, n_copy: int, n_content: int, gen: torch.Generator,
              device, far: bool = True) -> Tuple[torch.Tensor, torch.Tensor, int]:
    """Content tokens [0, n_content), marker n_content, separator
    n_content + 1, filler after those.  ``far``: the first copy opens the
    sequence and the filler sits between it and the separator (recall over
    about seq_len tokens); otherwise the filler comes first and the first
    copy ends right before the separator (recall over 3 n_copy tokens, inside
    the local window when 3 n_copy < sqrt(seq_len))."""
    mark, sep_tok, f0 = n_content, n_content + 1, n_content + 2
    vocab = f0 + N_FILL
    fill = seq_len - 3 * n_copy - 1
    if fill < 0:
        raise ValueError(f"seq_len {seq_len} too short for {n_copy} copied tokens")
    content = torch.randint(0, n_content, (n, n_copy), generator=gen, device=device)
    x = torch.randint(f0, vocab, (n, seq_len), generator=gen, device=device)
    tgt = torch.full((n, seq_len), -100, dtype=torch.long, device=device)
    c0 = 0 if far else fill
    x[:, c0:c0 + 2 * n_copy:2] = content
    x[:, c0 + 1:c0 + 2 * n_copy:2] = mark
    sep = 2 * n_copy + fill
    x[:, sep] = sep_tok
    x[:, sep + 1:sep + 1 + n_copy] = content
    # position p predicts token p + 1: the copy's tokens from the separator on
    tgt[:, sep:sep + n_copy] = content
    return x, tgt, vocab


class Block(nn.Module):
    def __init__(self, d: int, heads: int, attn: str):
        super().__init__()
        self.heads, self.attn = heads, attn
        self.n1 = nn.RMSNorm(d)
        self.qkv = nn.Linear(d, 3 * d, bias=False)
        self.proj = nn.Linear(d, d, bias=False)
        self.n2 = nn.RMSNorm(d)
        self.mlp = nn.Sequential(nn.Linear(d, 4 * d, bias=False), nn.GELU(), nn.Linear(4 * d, d, bias=False))

    def forward(self, x):
        B, S, d = x.shape
        q, k, v = self.qkv(self.n1(x)).view(B, S, 3, self.heads, d // self.heads).permute(2, 0, 3, 1, 4)
        if self.attn == "cra":
            from .core import cron_root_attention
            a = cron_root_attention(q, k, v)
        else:
            a = F.scaled_dot_product_attention(q, k, v, is_causal=True)
        x = x + self.proj(a.transpose(1, 2).reshape(B, S, d))
        return x + self.mlp(self.n2(x))


class TinyLM(nn.Module):
    def __init__(self, vocab: int, d: int, heads: int, layers: int, seq_len: int, attn: str):
        super().__init__()
        self.emb = nn.Embedding(vocab, d)
        self.pos = nn.Embedding(seq_len, d)
        self.blocks = nn.ModuleList(Block(d, heads, attn) for _ in range(layers))
        self.norm = nn.RMSNorm(d)
        self.head = nn.Linear(d, vocab, bias=False)

    def forward(self, x):
        h = self.emb(x) + self.pos(torch.arange(x.shape[1], device=x.device))
        for blk in self.blocks:
            h = blk(h)
        return self.head(self.norm(h))


def run(task: str = "mqar", attn: str = "cra", seq_len: int = 4096, steps: int = 400, batch: int = 16,
        d_model: int = 128, heads: int = 2, layers: int = 2, lr: float = 2e-3, seed: int = 0,
        n_eval: int = 256, n_kv: int = 16, n_queries: int = 8, device=None) -> dict:
    """Trains one model and returns its held-out accuracy on the scored
    positions (and the final training loss)."""
    device = device or torch.device("cuda", torch.cuda.current_device())
    gen = torch.Generator(device=device).manual_seed(seed)

    def data(n):
        if task == "mqar":
            return make_mqar(n, seq_len, n_kv=n_kv, n_queries=n_queries, gen=gen, device=device)
        return make_copy(n, seq_len, n_copy=n_queries, n_content=n_kv, gen=gen, device=device,
                         far=task == "copy")

    ex, et, vocab = data(n_eval)
    torch.manual_seed(seed)
    model = TinyLM(vocab, d_model, heads, layers, seq_len, attn).to(device)
    opt = torch.optim.AdamW(model.parameters(), lr=lr, weight_decay=0.0)
    sched = torch.optim.lr_scheduler.LambdaLR(opt, lambda s: min(1.0, (s + 1) / 50) * 0.5 *
                                              (1 + math.cos(math.pi * min(s, steps) / steps)))
    t0 = time.time()
    loss_v = float("nan")
    for step in range(steps):
        x, y, _ = data(batch)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            logits = model(x)
        loss = F.cross_entropy(logits.float().view(-1, vocab), y.view(-1), ignore_index=-100)
        opt.zero_grad(set_to_none=True)
        loss.backward()
        torch.nn.utils.clip_grad_norm_(model.parameters(), 1.0)
        opt.step()
        sched.step()
        loss_v = loss.item() if step % 50 == 0 or step == steps - 1 else loss_v
    model.eval()
    correct = total = 0
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
        for i in range(0, n_eval, batch):
            pred = model(ex[i:i + batch]).argmax(-1)
            m = et[i:i + batch] != -100
            correct += (pred[m] == et[i:i + batch][m]).sum().item()
            total += m.sum().item()
    return {"task": task, "attn": attn, "seq_len": seq_len, "steps": steps, "accuracy": correct / max(total, 1),
            "final_loss": loss_v, "seconds": time.time() - t0}


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--task", choices=["mqar", "copy", "copy_near", "all"], default="all")
    ap.add_argument("--attn", nargs="+", default=["sdpa", "cra"], choices=["sdpa", "cra"])
    ap.add_argument("--seq", type=int, default=4096)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--batch", type=int, default=16)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--lr", type=float, default=2e-3)
    a = ap.parse_args()
    for task in (["mqar", "copy", "copy_near"] if a.task == "all" else [a.task]):
        for attn in a.attn:
            print(json.dumps(run(task, attn, a.seq, a.steps, a.batch, lr=a.lr, seed=a.seed)), flush=True)


if __name__ == "__main__":
    main()
