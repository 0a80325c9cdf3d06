"""The sparse input embedding on the GPU: the embedding-bag kernels against the
oracle (plain and token-superposition bags), the sparse-row RMSProp kernel
against the reference's GramReaperSparse fixtures (duplicate rows, an empty
step), and the graph-replayed sparse step of HybridGraphOptimizer against the
eager one over several steps with a changing learning rate."""
import numpy as np
import pytest
import torch

from _util import rel_err
from oracle import sparse as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("shape", [(3, 17), (2, 9, 4)])
def test_embedding_bag_matches_oracle(shape):
    from zs_b200.lm import EmbeddingBagFunction

    torch.manual_seed(0)
    V, d = 101, 96
    table = torch.randn(V, d, device="cuda", requires_grad=True)
    ids = torch.randint(0, V, shape, device="cuda")
    out = EmbeddingBagFunction.apply(ids, table, 96 ** 0.5)
    ref = O.embedding_bag(table.detach().cpu().numpy(), ids.cpu().numpy(), 96 ** 0.5)
    assert rel_err(out, ref) < 1e-6
    dy = torch.randn_like(out)
    out.backward(dy)
    g = table.grad
    assert g.is_sparse
    rows, vals = O.embedding_bag_coo(dy.cpu().numpy(), ids.cpu().numpy(), 96 ** 0.5)
    assert torch.equal(g._indices()[0].cpu(), torch.as_tensor(rows))
    assert rel_err(g._values(), vals) < 1e-6
    # the same gradient as torch's own sparse embedding backward
    t2 = table.detach().clone().requires_grad_(True)
    e = torch.nn.functional.embedding(ids, t2, sparse=True)
    ref2 = (e.float().mean(dim=-2) if ids.dim() == 3 else e) * 96 ** 0.5
    ref2.backward(dy)
    assert rel_err(g.coalesce().to_dense(), t2.grad.coalesce().to_dense()) < 1e-6


@pytest.mark.parametrize("name,unit", [("sparse_unit", True), ("sparse_plain", False)])
def test_sparse_rmsprop_matches_reference(golden, name, unit):
    from engram.GramReaperSparse import GramReaperSparse
    from zs_b200 import device_error

    f = golden(name)
    p = torch.nn.Parameter(torch.tensor(f["W0"], device="cuda"))
    opt = GramReaperSparse([dict(params=[p], unit_norm=unit)], lr=3e-2, beta=0.9, unit_norm=unit)
    for k in range(3):
        rows = torch.tensor(f[f"rows{k}"], device="cuda")
        vals = torch.tensor(f[f"vals{k}"], device="cuda")
        p.grad = torch.sparse_coo_tensor(rows.view(1, -1), vals, tuple(p.shape))
        opt.step()
        np.testing.assert_allclose(p.detach().cpu().numpy(), f[f"W{k + 1}"], rtol=3e-6, atol=3e-7)
    st = opt.state[p]
    np.testing.assert_allclose(st["v"].cpu().numpy(), f["v"], rtol=3e-6, atol=1e-8)
    assert int(st["t"]) == int(f["t"]) == 2
    assert device_error() == 0


def test_sparse_step_large_table_matches_oracle():
    """A table with more than 2^16 rows (three radix passes), config-4 width, many duplicates."""
    from engram.GramReaperSparse import GramReaperSparse

    torch.manual_seed(1)
    V, d, n = 70001, 1536, 40000
    p = torch.nn.Parameter(torch.nn.functional.normalize(torch.randn(V, d, device="cuda"), dim=1))
    opt = GramReaperSparse([dict(params=[p], unit_norm=True)], lr=3e-3, beta=0.9, unit_norm=True)
    rows = torch.randint(0, V, (n,), device="cuda")
    rows[:500] = 7
    vals = torch.randn(n, d, device="cuda") * 0.01
    P = p.detach().cpu().numpy().copy()
    v = np.zeros(V, np.float32)
    p.grad = torch.sparse_coo_tensor(rows.view(1, -1), vals, (V, d))
    opt.step()
    O.sparse_rmsprop_step(P, v, 0, rows.cpu().numpy(), vals.cpu().numpy(), 3e-3, 0.9, 1e-10, True)
    touched = np.unique(rows.cpu().numpy())
    got = p.detach().cpu().numpy()
    np.testing.assert_allclose(got[touched], P[touched], rtol=2e-5, atol=2e-6)
    untouched = np.setdiff1d(np.arange(V), touched)
    assert np.array_equal(got[untouched], P[untouched])
    np.testing.assert_allclose(opt.state[p]["v"].cpu().numpy(), v, rtol=2e-5, atol=1e-9)


class _PlainSGD(torch.optim.Optimizer):
    """p -= lr * grad with no host work (recordable in a CUDA graph)."""

    def __init__(self, params, lr):
        super().__init__(params, dict(lr=lr))

    @torch.no_grad()
    def step(self, closure=None):
        for g in self.param_groups:
            for p in g["params"]:
                p.sub_(p.grad * g["lr"])


def test_hybrid_graph_replays_sparse_step_like_eager():
    from engram.GramReaperSparse import GramReaperSparse
    from optimizer.hybrid import HybridGraphOptimizer

    torch.manual_seed(2)
    V, d, n = 300, 64, 256

    def build():
        w = torch.nn.Parameter(torch.randn(32, 32, device="cuda"))
        t = torch.nn.Parameter(torch.nn.functional.normalize(torch.randn(V, d, device="cuda"), dim=1))
        dense = _PlainSGD([w], 0.1)
        sparse = GramReaperSparse([dict(params=[t], unit_norm=True)], lr=1e-2, beta=0.9, unit_norm=True)
        return w, t, dense, sparse

    w1, t1, d1, s1 = build()
    w2, t2, d2, s2 = build()
    with torch.no_grad():
        w2.copy_(w1)
        t2.copy_(t1)
    graphed = HybridGraphOptimizer(d1, s1, capture_warmup_steps=2)
    eager = HybridGraphOptimizer(d2, s2, capture_warmup_steps=2, enable_cuda_graph=False)
    g = torch.Generator(device="cuda").manual_seed(3)
    for step in range(6):
        rows = torch.randint(0, V, (n,), device="cuda", generator=g)
        vals = torch.randn(n, d, device="cuda", generator=g)
        gw = torch.randn(32, 32, device="cuda", generator=g)
        for opt, (w, t) in ((graphed, (w1, t1)), (eager, (w2, t2))):
            opt.zero_grad(set_to_none=False)
            if w.grad is None:
                w.grad = gw.clone()
            else:
                w.grad.copy_(gw)
            t.grad = torch.sparse_coo_tensor(rows.view(1, -1), vals.clone(), (V, d))
            for grp in opt.sparse.param_groups:
                grp["lr"] = 1e-2 * (1.0 - 0.1 * step)    # a float lr the scheduler changes
            opt.step()
        torch.cuda.synchronize()
        assert torch.equal(w1, w2), step
        assert torch.equal(t1, t2), step
    assert graphed._dense_graph is not None and len(graphed._sparse_graphs) == 1
    assert int(s1.state[t1]["t"]) == int(s2.state[t2]["t"]) == 6
