"""Forward + backward through the public API captured in one CUDA graph and
replayed: the library allocates nothing and never synchronizes inside its
calls (every buffer, the backward workspace included, comes from the
caller, here PyTorch's graph memory pool), so the replay gives the eager
results.  Replays with new inputs copied into the captured tensors must give
the new results."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("S,D,dt", [(4096, 128, torch.bfloat16), (1500, 64, torch.float16)])
def test_fwd_bwd_graph_replay_matches_eager(S, D, dt, cuda_device):
    import cron_root_attention as cra

    g = torch.Generator(device=cuda_device).manual_seed(S)
    B, H = 1, 4

    def draw():
        return [torch.randn(B, H, S, D, device=cuda_device, generator=g).to(dt) for _ in range(4)]

    def eager(q, k, v, do):
        qq, kk, vv = (t.detach().clone().requires_grad_(True) for t in (q, k, v))
        o = cra.cron_root_attention(qq, kk, vv)
        o.backward(do)
        return o.detach(), qq.grad, kk.grad, vv.grad

    sq, sk, sv, sdo = draw()
    sq, sk, sv = (t.requires_grad_(True) for t in (sq, sk, sv))
    side = torch.cuda.Stream(cuda_device)
    side.wait_stream(torch.cuda.current_stream(cuda_device))
    with torch.cuda.stream(side):  # warm-up outside the capture
        for _ in range(2):
            cra.cron_root_attention(sq, sk, sv).backward(sdo)
            sq.grad = sk.grad = sv.grad = None
    torch.cuda.current_stream(cuda_device).wait_stream(side)

    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        so = cra.cron_root_attention(sq, sk, sv)
        so.backward(sdo)
    gq, gk, gv = sq.grad, sk.grad, sv.grad

    for _ in range(2):  # the captured inputs, then new ones copied in
        graph.replay()
        torch.cuda.synchronize(cuda_device)
        ref = eager(sq.detach(), sk.detach(), sv.detach(), sdo)
        for a, b in zip((so.detach(), gq, gk, gv), ref):
            assert torch.equal(a, b)
        with torch.no_grad():
            for t, n in zip((sq, sk, sv, sdo), draw()):
                t.copy_(n)
    assert cra.check_device_errors(cuda_device) == 0
