"""Newton-Schulz split over data-parallel ranks and the Muon optimizer family, host
logic on CPU with two gloo ranks.  The Newton-Schulz function itself is replaced
by the oracle's CPU restatement (optimizer/muon.py:6-32) so the sharding, the
all-gather and the optimizers' arithmetic run without a GPU:

* _zeropower_many over two ranks returns, on every rank, exactly what one process
  returns for the same matrices (stacks, tall matrices, batches smaller than the
  world, mixed shapes and step counts);
* Muon / MuonWithAuxAdam on two ranks leave the parameters bit-identical to
  SingleDeviceMuon / SingleDeviceMuonWithAuxAdam in one process;
* SingleDeviceMuonWithAuxAdam follows the reference's update formula
  (optimizer/muon.py:35-42, :131-136, :266-300) step by step.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import muon as M


def _oracle_ns(X, steps):
    return torch.from_numpy(M.newton_schulz5(X.float().numpy(), steps=steps).astype(np.float32)).bfloat16()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _matrices():
    g = torch.Generator().manual_seed(5)
    shapes = [(3, 24, 40), (40, 24), (24, 40), (1, 16, 16), (5, 48, 16), (16, 16), (7, 8, 24)]
    return [torch.randn(s, generator=g) for s in shapes], [5, 5, 5, 3, 5, 3, 5]


def _params():
    g = torch.Generator().manual_seed(11)
    muon = [torch.nn.Parameter(torch.randn(s, generator=g) * 0.02) for s in [(32, 48), (4, 16, 24), (48, 32), (2, 3, 4, 4)]]
    adam = [torch.nn.Parameter(torch.randn(s, generator=g)) for s in [(48,), (16,)]]
    grads = [[torch.randn(p.shape, generator=g) for p in muon + adam] for _ in range(3)]
    return muon, adam, grads


def _run_opt(make, steps_grads, muon, adam):
    opt = make(muon, adam)
    for grads in steps_grads:
        for p, gr in zip(muon + adam, grads):
            p.grad = gr.clone()
        opt.step()
    return [p.detach().clone() for p in muon + adam]


def _single_muon(muon, adam):
    from optimizer.muon import SingleDeviceMuonWithAuxAdam

    return SingleDeviceMuonWithAuxAdam([dict(params=muon, use_muon=True, lr=0.02, weight_decay=0.01),
                                        dict(params=adam, use_muon=False, lr=1e-3, weight_decay=0.1)])


def _dist_muon(muon, adam):
    from optimizer.muon import MuonWithAuxAdam

    return MuonWithAuxAdam([dict(params=muon, use_muon=True, lr=0.02, weight_decay=0.01),
                            dict(params=adam, use_muon=False, lr=1e-3, weight_decay=0.1)])


def _worker(rank, world, port, q):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=__import__("datetime").timedelta(seconds=60))
        import optimizer.muon as OM

        OM.zeropower_via_newtonschulz5 = _oracle_ns
        Xs, steps = _matrices()
        single = OM._zeropower_many(Xs, steps)
        shard = OM._zeropower_many(Xs, steps, dist.group.WORLD)
        same = all(torch.equal(a, b) and a.shape == b.shape for a, b in zip(single, shard))

        muon, adam, grads = _params()
        ref = _run_opt(_single_muon, grads, muon, adam)
        muon, adam, grads = _params()
        got = _run_opt(_dist_muon, grads, muon, adam)
        same_opt = all(torch.equal(a, b) for a, b in zip(ref, got))

        from optimizer.muon import Muon, SingleDeviceMuon

        muon, _, grads = _params()
        ref1 = _run_opt(lambda m, a: SingleDeviceMuon(m, lr=0.05, weight_decay=0.0), [g[:4] for g in grads], muon, [])
        muon, _, grads = _params()
        got1 = _run_opt(lambda m, a: Muon(m, lr=0.05, weight_decay=0.0), [g[:4] for g in grads], muon, [])
        same_muon = all(torch.equal(a, b) for a, b in zip(ref1, got1))
        dist.destroy_process_group()
        q.put((rank, same, same_opt, same_muon, None))
    except Exception as e:  # pragma: no cover - reported to the parent
        import traceback

        q.put((rank, False, False, False, traceback.format_exc()))


def test_sharded_newton_schulz_and_muon_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=240) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, same, same_opt, same_muon, err in res:
        assert err is None, err
        assert same, f"rank {rank}: sharded Newton-Schulz differs from the single-process result"
        assert same_opt, f"rank {rank}: MuonWithAuxAdam differs from SingleDeviceMuonWithAuxAdam"
        assert same_muon, f"rank {rank}: Muon differs from SingleDeviceMuon"


def test_single_device_muon_with_aux_adam_follows_reference_formula(monkeypatch):
    import optimizer.muon as OM

    monkeypatch.setattr(OM, "zeropower_via_newtonschulz5", _oracle_ns)
    muon, adam, grads = _params()
    got = _run_opt(_single_muon, grads, muon, adam)

    # the reference's step, written out (optimizer/muon.py:35-42, :131-136, :266-300)
    muon, adam, grads = _params()
    mom = [torch.zeros_like(p) for p in muon]
    m1 = [torch.zeros_like(p) for p in adam]
    m2 = [torch.zeros_like(p) for p in adam]
    with torch.no_grad():
        for step, gs in enumerate(grads, 1):
            for i, p in enumerate(muon):
                g = gs[i].clone()
                mom[i].lerp_(g, 1 - 0.95)
                u = g.lerp_(mom[i], 0.95)
                if u.ndim == 4:
                    u = u.view(len(u), -1)
                u = _oracle_ns(u, 5)
                u *= max(1, g.size(-2) / g.size(-1)) ** 0.5
                p.mul_(1 - 0.02 * 0.01)
                p.add_(u.reshape(p.shape), alpha=-0.02)
            for i, p in enumerate(adam):
                g = gs[len(muon) + i]
                m1[i].lerp_(g, 1 - 0.9)
                m2[i].lerp_(g.square(), 1 - 0.95)
                upd = (m1[i] / (1 - 0.9 ** step)) / ((m2[i] / (1 - 0.95 ** step)).sqrt() + 1e-10)
                p.mul_(1 - 1e-3 * 0.1)
                p.add_(upd, alpha=-1e-3)
    for a, b in zip(got, muon + adam):
        assert torch.equal(a, b.detach())


def test_world_of_none_is_single_process():
    from optimizer.muon import _world

    assert _world(None) == (1, 0)
