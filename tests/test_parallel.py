"""Multi-rank host logic (gloo on CPU, world size 2 and 3): head/batch
sharding and the sequence split's exchange steps (global-row all-gather and
halo exchange) checked against the oracle on the whole sequence."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from cron_root_attention.parallel import seq_shard, shard_units, window


@pytest.mark.parametrize("B,H,world", [(1, 32, 8), (2, 16, 4), (1, 12, 5), (3, 7, 4), (1, 16, 1)])
def test_shard_units_partition(B, H, world):
    seen = []
    for r in range(world):
        for b, h0, h1 in shard_units(B, H, world, r):
            seen += [(b, h) for h in range(h0, h1)]
    assert sorted(seen) == [(b, h) for b in range(B) for h in range(H)]


@pytest.mark.parametrize("S,world,top_k", [(524288, 8, 2), (65536, 2, 2), (3000, 3, 2), (2049, 2, 2),
                                           (65536, 4, 4), (40000, 8, 1)])
def test_seq_shard_block_aligned_cover(S, world, top_k):
    W = window(S)
    prev = 0
    for r in range(world):
        b, e = seq_shard(S, world, r, top_k)
        assert b == prev and b % W == 0 and e > b
        prev = e
    assert prev == S
    # about equal attention work per rank: visible keys per query counted
    # independently (local window + strided and relay rows of earlier blocks)
    R = 1 + top_k if S > 2048 else 1
    def keys(m):
        ls = max(m - W + 1, 0)
        return min(m + 1, W) + R * (ls // W) + (ls % W != 0)
    work = [sum(keys(m) for m in range(*seq_shard(S, world, r, top_k))) for r in range(world)]
    block = max(sum(keys(m) for m in range(b, min(b + W, S))) for b in range(0, S, W))
    assert max(work) - sum(work) / world <= block
    if S == 524288:
        assert W == 725


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, S, out_dir, use_scale):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    for p in (root, os.path.join(root, "cron-root-attention_b200"), here):
        sys.path.insert(0, p)
    import torch.distributed as dist
    from cron_root_attention.parallel import seq_parallel_forward, seq_shard
    from shard_oracle import OracleShardOps
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    g = torch.Generator().manual_seed(7)
    q, k, v = (torch.randn(1, 2, S, 16, generator=g, dtype=torch.float64) for _ in range(3))
    b, e = seq_shard(S, world, rank)
    o = seq_parallel_forward(q[:, :, b:e], k[:, :, b:e], v[:, :, b:e], S, ops=OracleShardOps())
    torch.save(o, os.path.join(out_dir, f"o{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world,S", [(2, 3000), (3, 2600), (2, 1500)])
def test_seq_parallel_forward_gloo(world, S, tmp_path):
    from oracle import cra_oracle as O
    mp.spawn(_worker, args=(world, _free_port(), S, str(tmp_path), False), nprocs=world, join=True)
    o = torch.cat([torch.load(tmp_path / f"o{r}.pt") for r in range(world)], dim=2)
    g = torch.Generator().manual_seed(7)
    q, k, v = (torch.randn(1, 2, S, 16, generator=g, dtype=torch.float64) for _ in range(3))
    ref, _ = O.forward(q, k, v, dtype=torch.float64)
    assert (o - ref).abs().max().item() < 1e-10


@pytest.mark.parametrize("S", [3000, 1500])
def test_seq_parallel_forward_without_process_group(S):
    """No initialized process group: one rank holds the whole sequence and
    nothing is exchanged."""
    import torch.distributed as dist
    from cron_root_attention.parallel import seq_parallel_forward
    from oracle import cra_oracle as O
    from shard_oracle import OracleShardOps
    assert not (dist.is_available() and dist.is_initialized())
    g = torch.Generator().manual_seed(7)
    q, k, v = (torch.randn(1, 2, S, 16, generator=g, dtype=torch.float64) for _ in range(3))
    o = seq_parallel_forward(q, k, v, S, ops=OracleShardOps())
    ref, _ = O.forward(q, k, v, dtype=torch.float64)
    assert (o - ref).abs().max().item() < 1e-10


def test_relay_build_shard_rejects_wrong_scale_length():
    """A relay scale with the wrong number of kv heads is refused on the host,
    before anything reaches a kernel."""
    from cron_root_attention.parallel import LibcraShardOps
    k = torch.zeros(1, 2, 3000, 64, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="relay_log_scale"):
        LibcraShardOps().relay_build_shard(k, k, 3000, 0, True, 2, torch.zeros(3))


def _bwd_worker(rank, world, port, S, out_dir):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    for p in (root, os.path.join(root, "cron-root-attention_b200"), here):
        sys.path.insert(0, p)
    import torch.distributed as dist
    from cron_root_attention.parallel import seq_parallel_attention, seq_shard
    from shard_oracle import OracleShardOps
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    g = torch.Generator().manual_seed(8)
    q, k, v, do = (torch.randn(1, 2, S, 16, generator=g, dtype=torch.float64) for _ in range(4))
    b, e = seq_shard(S, world, rank)
    qs, ks, vs = (t[:, :, b:e].clone().requires_grad_(True) for t in (q, k, v))
    o = seq_parallel_attention(qs, ks, vs, S, ops=OracleShardOps())
    o.backward(do[:, :, b:e])
    torch.save((o.detach(), qs.grad, ks.grad, vs.grad), os.path.join(out_dir, f"g{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world,S", [(2, 3000), (3, 2600), (2, 1500)])
def test_seq_parallel_backward_gloo(world, S, tmp_path):
    """The sequence-split backward's exchanges -- dG summed over the ranks and
    folded into each rank's own blocks, halo gradients sent back to the
    previous rank -- give the whole sequence's gradients."""
    from oracle import cra_oracle as O
    mp.spawn(_bwd_worker, args=(world, _free_port(), S, str(tmp_path)), nprocs=world, join=True)
    parts = [torch.load(tmp_path / f"g{r}.pt") for r in range(world)]
    got = [torch.cat([p[i] for p in parts], dim=2) for i in range(4)]
    g = torch.Generator().manual_seed(8)
    q, k, v, do = (torch.randn(1, 2, S, 16, generator=g, dtype=torch.float64) for _ in range(4))
    ref = O.forward_backward(q, k, v, do, dtype=torch.float64)
    for x, y in zip(got, ref[:4]):
        assert (x - y).abs().max().item() < 1e-9
