"""Sequence split on the GPU: (a) every shard of a 2/3/8-way split run on one
GPU through the C ABI (cra_relay_build_shard + cra_fwd_shard) with the
exchange done in-process, against the oracle; (b) the real two-rank NCCL
path when two GPUs are present."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from oracle import cra_oracle as O
from parity import fwd_check, inputs

pytestmark = pytest.mark.gpu


def _emulate(q, k, v, S, world, dev, edge=True):
    """Every shard of a world-way split run on this GPU.  edge=True: each
    shard reads its own K / V rows in place plus a small edge copy (halo +
    first W + 256 rows), as the multi-GPU path does; edge=False: the halo
    rows placed in front of a copy of the shard."""
    from cron_root_attention.parallel import LibcraShardOps, seq_shard, window
    ops = LibcraShardOps()
    W = window(S)
    use_relay = S > 2048
    gks, gvs, outs = [], [], []
    bounds = [seq_shard(S, world, r) for r in range(world)]
    for b, e in bounds:
        gk, gv = ops.relay_build_shard(k[:, :, b:e].contiguous(), v[:, :, b:e].contiguous(), S, b, use_relay, 2, None)
        gks.append(gk)
        gvs.append(gv)
    gk, gv = torch.cat(gks, 2).contiguous(), torch.cat(gvs, 2).contiguous()
    for b, e in bounds:
        kb = max(0, b - (W - 1))
        if edge and b > 0:
            x = min(b + W + 256, e)
            eg = (k[:, :, kb:x].contiguous(), v[:, :, kb:x].contiguous(), kb)
            outs.append(ops.forward_shard(q[:, :, b:e].contiguous(), k[:, :, b:e].contiguous(),
                                          v[:, :, b:e].contiguous(), gk, gv, S, b, b, use_relay, 2, edge=eg))
        else:
            outs.append(ops.forward_shard(q[:, :, b:e].contiguous(), k[:, :, kb:e].contiguous(),
                                          v[:, :, kb:e].contiguous(), gk, gv, S, b, kb, use_relay, 2))
    torch.cuda.synchronize(dev)
    return torch.cat(outs, 2)


@pytest.mark.parametrize("S,world,D,dt,edge", [(5000, 2, 128, torch.bfloat16, True),
                                               (5000, 2, 128, torch.bfloat16, False),
                                               (9000, 3, 64, torch.float16, True),
                                               (40000, 8, 128, torch.bfloat16, True),
                                               (40000, 8, 128, torch.bfloat16, False)])
def test_sequence_split_emulated_on_one_gpu(S, world, D, dt, edge, cuda_device):
    q, k, v = inputs(1, 2, 2, S, D, dt, 50 + world)
    o = _emulate(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), S, world, cuda_device, edge)
    ref, _ = O.forward(q, k, v)
    r = fwd_check(o, ref, dt)
    assert r["ok"], r


def test_config5_shape_split_eight_ways(cuda_device):
    """BASELINE config 5's exact shape -- S = 524288 (W = 725, not a perfect
    square), D128 bf16, N(0,1), seed 4 (device generator) -- for two of its 16
    heads, split 8 ways as the 8-GPU run splits it, every shard run on this
    GPU, whole output checked row by row against the oracle."""
    dev = cuda_device
    S, H = 524288, 16
    g = torch.Generator(device=dev).manual_seed(4)
    q, k, v = (torch.randn(1, H, S, 128, generator=g, device=dev).to(torch.bfloat16) for _ in range(3))
    heads = [0, 9]
    q, k, v = (t[:, heads].contiguous() for t in (q, k, v))
    from cron_root_attention.parallel import window
    assert window(S) == 725
    o = _emulate(q, k, v, S, 8, dev)
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    for i in range(len(heads)):
        sl = lambda t: t[:, i:i + 1].cpu()
        ref, _ = O.forward(sl(q), sl(k), sl(v))
        r = fwd_check(sl(o), ref, torch.bfloat16)
        assert r["ok"], (heads[i], r)


def _emulate_bwd(q, k, v, do, S, world, dev):
    """The sequence-split backward of a world-way split, every shard on this
    GPU: the forward per shard, phase 1 per shard, dG summed over the shards
    (what the all-reduce does), phase 2 per shard, halo gradients added to the
    previous shard."""
    from cron_root_attention.parallel import LibcraShardOps, seq_shard, window
    ops = LibcraShardOps()
    W = window(S)
    use_relay = S > 2048
    bounds = [seq_shard(S, world, r) for r in range(world)]
    gks, gvs, srcs = [], [], []
    for b, e in bounds:
        gk, gv, src = ops.relay_build_shard(k[:, :, b:e].contiguous(), v[:, :, b:e].contiguous(), S, b, use_relay, 2,
                                            None, with_src=True)
        gks.append(gk), gvs.append(gv), srcs.append(src)
    gk, gv, gsrc = (torch.cat(x, 2).contiguous() for x in (gks, gvs, srcs))
    st = []
    for b, e in bounds:
        sl = lambda t: t[:, :, b:e].contiguous()
        edge = None
        if b > 0:
            kb = max(0, b - (W - 1))
            x = min(b + W + 256, e)
            edge = (k[:, :, kb:x].contiguous(), v[:, :, kb:x].contiguous(), kb)
        o, lse = ops.forward_shard(sl(q), sl(k), sl(v), gk, gv, S, b, b if b > 0 else 0, use_relay, 2, edge=edge,
                                   return_lse=True)
        dgk, dgv, ws = ops.backward_global(sl(q), o, sl(do), lse, gk, gv, S, b, use_relay, 2)
        st.append((b, e, edge, o, dgk, dgv, ws))
    dgk = sum(x[4] for x in st)
    dgv = sum(x[5] for x in st)
    dqs, dks, dvs, halos = [], [], [], []
    for b, e, edge, o, _, _, ws in st:
        sl = lambda t: t[:, :, b:e].contiguous()
        dq, dk, dv, dkh, dvh, _ = ops.backward_local(sl(q), sl(k), sl(v), sl(do), gk, gv, gsrc, dgk, dgv, ws, S, b,
                                                     use_relay, 2, edge, None)
        dqs.append(dq), dks.append(dk), dvs.append(dv), halos.append((dkh, dvh))
    for r in range(1, world):
        dkh, dvh = halos[r]
        n = dkh.shape[2]
        dks[r - 1][:, :, -n:] += dkh
        dvs[r - 1][:, :, -n:] += dvh
    torch.cuda.synchronize(dev)
    return torch.cat(dqs, 2), torch.cat(dks, 2), torch.cat(dvs, 2)


@pytest.mark.parametrize("S,world,D,dt", [(5000, 2, 128, torch.bfloat16), (9000, 3, 64, torch.float16),
                                          (40000, 8, 128, torch.bfloat16), (1800, 2, 128, torch.float16)])
def test_sequence_split_backward_emulated_on_one_gpu(S, world, D, dt, cuda_device):
    """Gradients of a sequence split across `world` shards (libcra's two shard
    phases) against the fp64 oracle of the whole sequence."""
    from parity import GRAD_REL_L2, rel_l2
    import cron_root_attention as cra
    q, k, v, do = inputs(1, 2, 2, S, D, dt, 80 + world, with_do=True)
    dev = cuda_device
    dq, dk, dv = _emulate_bwd(*(t.to(dev) for t in (q, k, v, do)), S, world, dev)
    assert cra.check_device_errors(dev) == 0
    _, rdq, rdk, rdv, _ = O.forward_backward(q, k, v, do)
    for name, x, y in (("dq", dq, rdq), ("dk", dk, rdk), ("dv", dv, rdv)):
        assert rel_l2(x, y) <= GRAD_REL_L2, (name, rel_l2(x, y))


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _nccl_worker(rank, world, port, S, out):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    for p in (root, os.path.join(root, "cron-root-attention_b200"), here):
        sys.path.insert(0, p)
    import torch.distributed as dist
    from cron_root_attention.parallel import seq_parallel_forward, seq_shard
    from parity import inputs
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world)
    q, k, v = inputs(1, 2, 2, S, 128, torch.bfloat16, 60)
    b, e = seq_shard(S, world, rank)
    dev = torch.device("cuda", rank)
    o = seq_parallel_forward(q[:, :, b:e].to(dev), k[:, :, b:e].to(dev), v[:, :, b:e].to(dev), S)
    torch.save(o.cpu(), os.path.join(out, f"o{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


def _nccl_bwd_worker(rank, world, port, S, out):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    for p in (root, os.path.join(root, "cron-root-attention_b200"), here):
        sys.path.insert(0, p)
    import torch.distributed as dist
    from cron_root_attention.parallel import seq_parallel_attention, seq_shard
    from parity import inputs
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world)
    q, k, v, do = inputs(1, 2, 2, S, 128, torch.bfloat16, 61, with_do=True)
    b, e = seq_shard(S, world, rank)
    dev = torch.device("cuda", rank)
    qs, ks, vs = (t[:, :, b:e].to(dev).requires_grad_(True) for t in (q, k, v))
    o = seq_parallel_attention(qs, ks, vs, S)
    o.backward(do[:, :, b:e].to(dev))
    torch.save(tuple(t.cpu() for t in (qs.grad, ks.grad, vs.grad)), os.path.join(out, f"g{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_sequence_split_backward_nccl_two_ranks(tmp_path):
    from parity import GRAD_REL_L2, rel_l2
    S = 12000
    mp.spawn(_nccl_bwd_worker, args=(2, _port(), S, str(tmp_path)), nprocs=2, join=True)
    parts = [torch.load(tmp_path / f"g{r}.pt") for r in range(2)]
    got = [torch.cat([p[i] for p in parts], 2) for i in range(3)]
    q, k, v, do = inputs(1, 2, 2, S, 128, torch.bfloat16, 61, with_do=True)
    _, rdq, rdk, rdv, _ = O.forward_backward(q, k, v, do)
    for name, x, y in zip(("dq", "dk", "dv"), got, (rdq, rdk, rdv)):
        assert rel_l2(x, y) <= GRAD_REL_L2, (name, rel_l2(x, y))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_sequence_split_nccl_two_ranks(tmp_path):
    S = 12000
    mp.spawn(_nccl_worker, args=(2, _port(), S, str(tmp_path)), nprocs=2, join=True)
    o = torch.cat([torch.load(tmp_path / f"o{r}.pt") for r in range(2)], 2)
    q, k, v = inputs(1, 2, 2, S, 128, torch.bfloat16, 60)
    ref, _ = O.forward(q, k, v)
    r = fwd_check(o, ref, torch.bfloat16)
    assert r["ok"], r
