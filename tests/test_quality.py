"""The model-quality check (cron_root_attention.quality): task generators on
the CPU, and a short training run of the same small model with this
package's attention and with dense causal attention on the GPU."""
import pytest
import torch

from cron_root_attention import quality as Q


def test_mqar_generator():
    g = torch.Generator().manual_seed(0)
    x, t, vocab = Q.make_mqar(4, 200, n_kv=8, n_queries=3, gen=g, device="cpu")
    assert x.shape == t.shape == (4, 200) and vocab == 18 + Q.N_FILL
    # a key token appears only in the pair region and in the queries
    sep = 200 - 3 * 2
    assert not ((x[:, 16:sep] >= 2) & (x[:, 16:sep] < 10)).any()
    for i in range(4):
        kv = {int(x[i, 2 * j]): int(x[i, 2 * j + 1]) for j in range(8)}  # key token -> value token
        pos = (t[i] != -100).nonzero().flatten().tolist()
        assert len(pos) == 3
        for p in pos:
            assert x[i, p] == 1 and int(t[i, p]) == kv[int(x[i, p - 1])]


def test_copy_generator():
    g = torch.Generator().manual_seed(1)
    x, t, vocab = Q.make_copy(3, 120, n_copy=5, n_content=10, gen=g, device="cpu")
    assert vocab == 12 + Q.N_FILL
    for i in range(3):
        content = x[i, 0:10:2]
        pos = (t[i] != -100).nonzero().flatten()
        assert len(pos) == 5 and torch.equal(t[i, pos], content)
        assert torch.equal(x[i, pos + 1], content)  # position p predicts token p + 1
        assert x[i, pos[0]] == 11


def test_copy_near_generator():
    g = torch.Generator().manual_seed(2)
    x, t, _ = Q.make_copy(2, 120, n_copy=5, n_content=10, gen=g, device="cpu", far=False)
    sep = 120 - 5 - 1
    assert torch.equal(x[:, sep - 10:sep:2], t[:, sep:sep + 5])  # first copy ends at the separator


@pytest.mark.gpu
def test_local_recall_is_learned(cuda_device):
    """Copy inside the local window (S = 2304, W = 48, recall distance <= 24):
    every key a recall position needs is in its sparse pattern, and a model
    trained through this package's forward and backward kernels learns the
    task (alone, seeds 0, 1 and 2 reached 1.0 at 2000 steps on B200; after
    the other GPU tests the same seed reached 0.88: training is not
    bit-reproducible across processes, so the bar is well above chance,
    1 / 16, rather than exact recall)."""
    r = Q.run("copy_near", "cra", seq_len=2304, steps=2000, batch=16, lr=1e-3, seed=1, n_eval=64,
              device=cuda_device)
    assert r["accuracy"] > 0.5, r


@pytest.mark.gpu
def test_far_recall_runs(cuda_device):
    """Far copy (recall over about S tokens) trains and evaluates through the
    sparse kernels with a finite loss; its accuracy is reported, not bounded
    (the pattern reaches far keys only through strided and relay keys)."""
    r = Q.run("copy", "cra", seq_len=2304, steps=100, batch=16, seed=0, n_eval=32, device=cuda_device)
    assert r["final_loss"] == r["final_loss"] and 0.0 <= r["accuracy"] <= 1.0
