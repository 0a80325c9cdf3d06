"""Data-parallel host logic on CPU with two gloo ranks: the bucketed, hook-driven
gradient all-reduce (dense, sparse embedding, gradients written outside autograd,
mixed dtypes, bucket rebuild after the first step) and the routing-count
all-reduce behind the aux-loss-free bias update (main.py:161-175)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=__import__("datetime").timedelta(seconds=60))


class _OutsideAutograd(torch.autograd.Function):
    """y = x @ W^T whose backward adds dW into W.grad itself and returns None for W
    (the fused expert weight-gradient pattern)."""

    @staticmethod
    def forward(ctx, x, W):
        ctx.save_for_backward(x)
        ctx.W = W
        return x @ W.t()

    @staticmethod
    def backward(ctx, dy):
        (x,) = ctx.saved_tensors
        W = ctx.W
        g = dy.reshape(-1, dy.size(-1)).t() @ x.reshape(-1, x.size(-1))
        if W.grad is None:
            W.grad = g
        else:
            W.grad += g
        from zs_b200.dp import notify_grad_ready

        notify_grad_ready(W)
        return dy @ W, None


class _Model(torch.nn.Module):
    def __init__(self):
        super().__init__()
        torch.manual_seed(0)
        self.emb = torch.nn.Embedding(50, 16, sparse=True)
        self.a = torch.nn.Linear(16, 32)
        self.W = torch.nn.Parameter(torch.randn(24, 32) * 0.1)
        self.b = torch.nn.Linear(24, 8).to(torch.float64)

    def forward(self, ids):
        h = torch.tanh(self.a(self.emb(ids)))
        h = _OutsideAutograd.apply(h, self.W)
        return self.b(h.double()).pow(2).mean()


def _grads(model):
    out = {}
    for n, p in model.named_parameters():
        g = p.grad
        out[n] = (g.to_dense() if g.is_sparse else g).clone()
    return out


def _reducer_worker(rank, world, port, q):
    try:
        _reducer_body(rank, world, port, q)
    except Exception as e:  # report instead of leaving the parent waiting
        q.put((rank, repr(e), None))
        raise


def _reducer_body(rank, world, port, q):
    from zs_b200.dp import GradAllReducer

    _init(rank, world, port)
    try:
        model = _Model()
        red = GradAllReducer(list(model.parameters()), bucket_mb=0.001, average=True)
        gen = torch.Generator().manual_seed(123)
        results = []
        for step in range(2):
            ids_all = torch.randint(0, 50, (world, 6, 5), generator=gen)
            model.zero_grad(set_to_none=True)
            model(ids_all[rank]).backward()
            red.finish()
            mine = _grads(model)
            # reference: the mean over ranks of the per-rank gradients, computed locally
            ref = _Model()
            ref.load_state_dict(model.state_dict())
            acc = None
            for r in range(world):
                ref.zero_grad(set_to_none=True)
                ref(ids_all[r]).backward()
                g = _grads(ref)
                acc = g if acc is None else {k: acc[k] + g[k] for k in acc}
            results.append(max(float((mine[k] - acc[k] / world).abs().max()) for k in acc))
        q.put((rank, results, red._rebuilt))
    finally:
        dist.destroy_process_group()


def _counts_worker(rank, world, port, q):
    try:
        _counts_body(rank, world, port, q)
    except Exception as e:
        q.put((rank, repr(e), None, None))
        raise


def _counts_body(rank, world, port, q):
    from oracle import routing as R
    from zs_b200.dp import all_reduce_counts

    _init(rank, world, port)
    try:
        E, k = 16, 4
        rng = np.random.default_rng(7)
        topk = [np.stack([rng.permutation(E)[:k] for _ in range(100 + 37 * r)]) for r in range(world)]
        local = torch.from_numpy(np.bincount(topk[rank].ravel(), minlength=E)).long().view(1, E)
        all_reduce_counts(local, dist.group.WORLD)
        glob = np.bincount(np.concatenate(topk).ravel(), minlength=E)
        bias0 = np.linspace(-0.1, 0.1, E).astype(np.float32)
        # the bias update every rank applies from the reduced counts ...
        counts = local[0].numpy().astype(np.float32)
        mean = np.float32(counts.sum(dtype=np.float32) * np.float32(np.float32(1.0) / np.float32(E)))
        mine = (bias0 + np.float32(1e-3) * np.sign((mean - counts).astype(np.float32))).astype(np.float32)
        # ... equals the single-process update on the global batch
        ref = R.aux_loss_free_update(bias0, np.concatenate(topk), 1e-3)
        q.put((rank, bool(np.array_equal(local[0].numpy(), glob)), bool(np.array_equal(mine, ref)), mine.tobytes()))
    finally:
        dist.destroy_process_group()


def _run(worker, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=90) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    return sorted(out)


def test_grad_all_reducer_two_ranks():
    out = _run(_reducer_worker)
    for rank, errs, rebuilt in out:
        assert rebuilt is True, errs
        assert all(e < 1e-6 for e in errs), (rank, errs)


def test_routing_counts_all_reduce_two_ranks():
    out = _run(_counts_worker)
    assert all(ok_counts and ok_bias for _, ok_counts, ok_bias, _ in out)
    assert out[0][3] == out[1][3]   # identical bias on both ranks


def test_copy_engine_peer_timeout_raises_and_drops_state(monkeypatch):
    """finish() after a copy-engine all-reduce reads the device error word: an expired
    peer wait (ZS_DEVERR_TIMEOUT_PEER) raises, and the copy-engine instances (whose step
    flags no longer agree with the peers') are closed and dropped (fake error word)."""
    from zs_b200 import _lib, dp

    r = dp.GradAllReducer.__new__(dp.GradAllReducer)
    closed = []

    class FakeCE:
        def close(self):
            closed.append(True)

    r._ce = {(0, torch.float32): FakeCE(), (1, torch.float32): FakeCE()}
    r._ce_used = True
    r.buckets = [[], []]
    monkeypatch.setattr(_lib, "device_error", lambda device=None: 0x20)
    monkeypatch.setattr(_lib, "clear_device_error", lambda device=None: None)
    with pytest.raises(RuntimeError, match="TIMEOUT_PEER"):
        r._check_peers()
    assert len(closed) == 2 and r._ce == {} and not r._ce_used
    # a clean error word passes
    r._ce_used = True
    monkeypatch.setattr(_lib, "device_error", lambda device=None: 0)
    r._check_peers()
